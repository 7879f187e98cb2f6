#pragma once
// Forward convolution as an implicit GEMM on the sm_100a tensor cores.
//
//   GEMM M = output pixels (a 128-pixel tile: tn images × th rows × tw columns, or 128 consecutive rows
//            of the [N·H·W, C] matrix for 1×1 convs), GEMM N = output channels (BN per tile),
//   GEMM K = taps × input channels, walked as (tap, BK-channel chunk) steps.
//
// Persistent kernel: each CTA walks the tile list (tile = blockIdx.x + i·gridDim.x, output-channel tile
// fastest so neighbouring CTAs share their A windows in L2).  Two CTAs per SM with 6 warps each when
// BN ≤ 128, one CTA with 10 warps for wider tiles:
//   warp 0      TMA producer: per K-step one A box (the input window of this tap, halo = TMA zero fill)
//               and one B box (KRSC weight rows) into a STAGES-deep ring; it runs ahead across tiles;
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer (M=128, N=BN, K=16), accumulating into
//               one of TWO TMEM buffers, so the MMAs of tile i+1 overlap the epilogue of tile i;
//   warps 2..   epilogue: one (BN ≤ 128) or two (wider, each taking half of the columns) warps per TMEM
//               lane quadrant:
//               tcgen05.ld, folded BN + SiLU (+ residual) or bias, fp16 conversion and the
//               multi-destination store (channel slices, 2× nearest upsample) — written back through a
//               per-warp shared-memory stage so that each store instruction covers whole pixel rows
//               (epilogue.cuh).  This replaces the reference's separate bn_forward_apply / add_bias passes.
// Operand tiles are K-major with the TMA swizzle (128 B rows for BK = 64, 64 B rows for BK = 32) the UMMA
// shared-memory descriptor expects.  No multicast anywhere.  Every wait is bounded (sm100.cuh).
//
// A_W3 (3×3, stride 1, pad 1; tiles of th rows × tw columns × ni images, th·tw·ni = 128, tw·ni ∈ {8, 16}):
// per BK-channel chunk the producer loads three column-shifted input windows ((th + 2) rows × ni images ×
// tw columns, shifts −1, 0, +1; a (C, W, N, H) view so a window's pixel rows run (row, image, column))
// instead of nine tap boxes.  The tile's GEMM rows run in the same (row, image, column) order, so tap
// (r, c) reads window c from pixel row r·ni·tw on — a whole number of swizzle atoms — and its UMMA
// descriptor is the plain K-major one.  The windows have their own ring; a window is released
// after its three taps.  A third of the A boxes and ~40 % of the A bytes of the per-tap form.
//
// A_W3R: the window form for narrow layers (C = BK, one N tile, BN ≤ 64): the nine weight taps are loaded
// once per CTA and stay in shared memory; per tile only the three windows stream.
//
// A_W3S2 / A_W3S2R: the window form of a 3×3 / stride-2 / pad-1 conv on 16 × 8 output tiles.  Through the
// parity view (2C, W/2, 2, H/2, N) a column tap dc ∈ {−1, 0, 1} is one box of 17 row pairs × both row
// parities × 8 columns (channel half dc & 1, column offset dc >> 1): pixel rows run (row pair, parity,
// column), so output row i of row tap r starts at pixel row 16·i + 8·(r + 1) — 8-row core groups 16 rows
// apart (SBO = 16 rows), each a whole swizzle atom.
//
// PAIR (CTA pairs on two SMs, cluster of 2): a work unit is two 128-pixel M tiles × BN channels, one
// tile per CTA, computed by 2-SM UMMAs (M = 256) that the leader CTA (rank 0) issues.  Each CTA stages
// its own A tile and HALF of the B (weight) rows.  Both producers' loads count on the leader's full
// barrier (the leader expects both CTAs' bytes); the leader's commits arrive on both CTAs' empty and
// accumulator barriers; both CTAs' epilogue warps arrive on the leader's drained barrier.
// The kernel template and its launchers; conv_fprop_n*.cu instantiate launch_mode<BK, BN> for the GEMM N
// tile widths (one translation unit per group, so the widths compile in parallel), conv_fprop.cu picks one.
#include "epilogue.cuh"

namespace osam {

constexpr int kMaxGemmN = 512;  // per-column epilogue constants cached in shared memory

template <int BK, int BN, bool PAIR, int MODE>
struct FpropCfg {
  static constexpr bool W3 = mode_window(MODE), RESB = mode_resident(MODE), S2W = mode_s2_window(MODE);
  static constexpr int A_BYTES = W3 ? 0 : 128 * BK * 2;  // per-tap A box in the joint ring (not with W3)
  static constexpr int B_ROWS = PAIR ? BN / 2 : BN;  // weight rows staged by this CTA
  static constexpr int B_BYTES = B_ROWS * BK * 2;
  static_assert(B_BYTES % 1024 == 0, "weight stages must keep the ring 1024-byte aligned");
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // ≤ 128 output channels: two CTAs per SM, each with 4 epilogue warps (two independent load/MMA
  // pipelines hide TMA latency better); wider tiles: one CTA per SM with 8 epilogue warps.
  // (one CTA per SM for the 128-wide window form, 8 epilogue warps and a 196 KB ring: measured 30 % slower)
  static constexpr bool ONE_CTA = BN > 128;
  static constexpr int CTAS_PER_SM = ONE_CTA ? 1 : 2;
  static constexpr int EPI_WARPS = ONE_CTA ? 8 : 4;
  static constexpr int RING_BUDGET = ONE_CTA ? 196 * 1024 : 96 * 1024;
  // A_W3 window ring: windows of (th + 2)·ni·tw ≤ 160 pixel rows; as many as fit (2…4) beside five weight
  // stages (the window loads are the latency-critical ones — a window feeds only three taps — but fewer
  // than five weight stages cost more than a deeper window ring gains: measured with 3, 5 and 7)
  static constexpr int W3_MIN_B = 5;
  static constexpr int WIN_ROWS = S2W ? 272 : 160;  // 17 row pairs × 2 parities × 8, or (th + 2)·ni·tw
  static constexpr int WIN_BYTES = W3 ? WIN_ROWS * BK * 2 : 0;
  static constexpr int A_FIT = W3 ? (RING_BUDGET - (RESB ? 9 : W3_MIN_B) * B_BYTES) / WIN_BYTES : 0;
  // resident-weight forms stream only windows: a deeper window ring (up to 8) keeps more loads in flight
  static constexpr int A_MAX = RESB ? 8 : 4;
  static constexpr int A_STAGES = W3 ? (A_FIT < 2 ? 2 : (A_FIT > A_MAX ? A_MAX : A_FIT)) : 0;
  static constexpr int STAGES_RAW = (RING_BUDGET - A_STAGES * WIN_BYTES) / STAGE_BYTES;
  // RESB: the nine weight taps, loaded once (full[0] counts them)
  static constexpr int STAGES = RESB ? 9 : (STAGES_RAW < 2 ? 2 : (STAGES_RAW > 8 ? 8 : STAGES_RAW));
  static constexpr int ACC_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static constexpr int TMEM_COLS = 2 * ACC_COLS;  // double-buffered accumulator
  static constexpr int ROW_BYTES = BK * 2;
  static constexpr int CONST_BYTES = 2 * kMaxGemmN * 4;
  static constexpr int STAGE_OUT_BYTES = EPI_WARPS * 32 * 64;  // per-warp epilogue stage
  static constexpr int SMEM_BYTES =
      1024 + A_STAGES * WIN_BYTES + STAGES * STAGE_BYTES + STAGE_OUT_BYTES + CONST_BYTES + 256;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
};

template <int BK, int BN, int MODE, bool PAIR = false>
__global__ void __launch_bounds__(FpropCfg<BK, BN, PAIR, MODE>::THREADS, FpropCfg<BK, BN, PAIR, MODE>::CTAS_PER_SM)
    k_conv_fprop(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                 const __grid_constant__ StoreMaps sm, const ConvDev d) {
  using Cfg = FpropCfg<BK, BN, PAIR, MODE>;
  constexpr bool W3 = Cfg::W3, RESB = Cfg::RESB, S2W = Cfg::S2W;
  constexpr int STAGES = Cfg::STAGES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = base;  // per-tap A boxes, or (A_W3) the window ring
  uint8_t* sB = base + (W3 ? Cfg::A_STAGES * Cfg::WIN_BYTES : STAGES * Cfg::A_BYTES);
  uint8_t* s_stage = sB + STAGES * Cfg::B_BYTES;  // 1024-aligned: the TMA store swizzle needs 512
  float* s_sc = reinterpret_cast<float*>(s_stage + Cfg::STAGE_OUT_BYTES);
  float* s_sh = s_sc + kMaxGemmN;
  uint64_t* full = reinterpret_cast<uint64_t*>(s_sh + kMaxGemmN);
  uint64_t* empty = full + STAGES;
  uint64_t* accf = empty + STAGES;  // [2] accumulator ready (MMA → epilogue)
  uint64_t* acce = accf + 2;        // [2] accumulator drained (epilogue → MMA), one arrival per epilogue warp
  uint64_t* afull = acce + 2;       // A_W3: [A_STAGES] window landed
  uint64_t* aempty = afull + Cfg::A_STAGES;  // A_W3: [A_STAGES] window's three taps consumed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(aempty + Cfg::A_STAGES);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // PAIR: units of two M tiles (this CTA's is 2·unit + rank), walked by cluster; else single tiles by CTA.
  const uint32_t rank = PAIR ? cluster_ctarank() : 0;
  const int ntiles = PAIR ? ((d.tiles_m + 1) >> 1) * d.ntn : d.tiles_m * d.ntn;
  const int t_first = PAIR ? (int)(blockIdx.x >> 1) : (int)blockIdx.x;
  const int t_step = PAIR ? (int)(gridDim.x >> 1) : (int)gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      mbar_init(full + s, 1);
      mbar_init(empty + s, 1);
    }
    for (int b = 0; b < 2; b++) {
      mbar_init(accf + b, 1);
      mbar_init(acce + b, (PAIR ? 2 : 1) * Cfg::EPI_WARPS);
    }
    for (int s = 0; s < Cfg::A_STAGES; s++) {
      mbar_init(afull + s, 1);
      mbar_init(aempty + s, 1);
    }
    fence_barrier_init();
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
  }
  if (warp == 1) {
    if (PAIR) {
      tmem_alloc_pair(tslot, Cfg::TMEM_COLS);
      tmem_relinquish_pair();
    } else {
      tmem_alloc(tslot, Cfg::TMEM_COLS);
      tmem_relinquish();
    }
  }
  // PAIR: both CTAs' barriers are initialised before either CTA signals the other's
  if (PAIR) {
    __syncwarp();  // the cluster barrier is warp-aligned
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  tc_fence_after();
  const uint32_t tmem = *tslot;
  // Programmatic dependent launch: the set-up above (barriers, TMEM, tensor-map prefetch) overlapped the
  // previous kernel's tail; the producer and the epilogue — the only threads touching global memory —
  // wait for that kernel below, and the next conv may begin its own set-up now.
  grid_dep_launch();

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) grid_dep_wait();
    if constexpr (W3) {
      if (lane == 0) {
        uint32_t it = 0, ait = 0;
        bool ok = true;
        const int tw = d.tw, th = d.th, ni = d.tn;
        const uint32_t wbytes = (uint32_t)((S2W ? 2 * (th + 1) : th + 2) * ni * tw * BK * 2);
        if (RESB) {  // the nine weight taps (this CTA's rows), once; full[0] counts them
          const int nb = (int)rank * Cfg::B_ROWS;
          if (PAIR) {
            if (rank == 0) mbar_arrive_expect_tx(full, 2 * 9 * Cfg::B_BYTES);
            for (int tap = 0; tap < 9; tap++)
              tma_load_2d_cg2(sB + tap * Cfg::B_BYTES, &tb, mapa_shared(full, 0), tap * d.C, nb);
          } else {
            mbar_arrive_expect_tx(full, 9 * Cfg::B_BYTES);
            for (int tap = 0; tap < 9; tap++) tma_load_2d(sB + tap * Cfg::B_BYTES, &tb, full, tap * d.C, nb);
          }
        }
        for (int t = t_first; t < ntiles && ok; t += t_step) {
          // PAIR: this CTA's tile of the unit (past the end for the peer of an odd last unit: zero fill),
          // its half of the weight rows; every load counts on the leader's barriers
          const int tn_q = d.f_ntn.quo(t), nt = d.f_ntn.rem(t, tn_q), mt = PAIR ? tn_q * 2 + (int)rank : tn_q;
          const int n0 = nt * BN + (int)rank * Cfg::B_ROWS;
          const int rest = d.f_tq.quo(mt), tq = d.f_tq.rem(mt, rest);
          const int rp = d.f_tp.quo(rest);
          const int q0 = tq * tw, p0 = d.f_tp.rem(rest, rp) * th, b0 = rp * ni;
          for (int cc = 0; cc < d.C && ok; cc += BK) {
            for (int c = 0; c < 3 && ok; c++, ait++) {
              const int ws = ait % Cfg::A_STAGES;
              if (ait >= (uint32_t)Cfg::A_STAGES && !mbar_wait(aempty + ws, ((ait / Cfg::A_STAGES) - 1) & 1, d.err)) {
                ok = false;
                break;
              }
              // window c: rows p0−1 … p0+th, images b0 … b0+ni−1, columns q0+c−1 … q0+c−2+tw (zero fill
              // outside the batch and the image); the map's dimensions are (C, W, N, H)
              // stride 2 (parity view): channel half dc & 1, column offset dc >> 1, both row parities, row
              // pairs p0−1 … p0+th−1
              const int dc = c - 1;
              uint8_t* wdst = sA + ws * Cfg::WIN_BYTES;
              if (PAIR) {
                if (rank == 0) mbar_arrive_expect_tx(afull + ws, 2 * wbytes);
                const uint32_t fb = mapa_shared(afull + ws, 0);
                if (S2W)
                  tma_load_5d_cg2(wdst, &ta, fb, (dc & 1) * d.C + cc, q0 + (dc >> 1), 0, p0 - 1, b0);
                else
                  tma_load_4d_cg2(wdst, &ta, fb, cc, q0 + c - 1, b0, p0 - 1);
              } else {
                mbar_arrive_expect_tx(afull + ws, wbytes);
                if (S2W)
                  tma_load_5d(wdst, &ta, afull + ws, (dc & 1) * d.C + cc, q0 + (dc >> 1), 0, p0 - 1, b0);
                else
                  tma_load_4d(wdst, &ta, afull + ws, cc, q0 + c - 1, b0, p0 - 1);
              }
              for (int r = 0; r < 3 && !RESB; r++, it++) {
                const int s = it % STAGES;
                if (it >= STAGES && !mbar_wait(empty + s, ((it / STAGES) - 1) & 1, d.err)) {
                  ok = false;
                  break;
                }
                if (PAIR) {
                  if (rank == 0) mbar_arrive_expect_tx(full + s, 2 * Cfg::B_BYTES);
                  tma_load_2d_cg2(sB + s * Cfg::B_BYTES, &tb, mapa_shared(full + s, 0), (r * 3 + c) * d.C + cc, n0);
                } else {
                  mbar_arrive_expect_tx(full + s, Cfg::B_BYTES);
                  tma_load_2d(sB + s * Cfg::B_BYTES, &tb, full + s, (r * 3 + c) * d.C + cc, n0);
                }
              }
            }
          }
        }
        // PAIR: the leader's last commits arrive on this CTA's barriers; wait for them before retiring
        if (PAIR && ok) {
          for (uint32_t j = it > (uint32_t)STAGES ? it - STAGES : 0; j < it; j++)
            if (!mbar_wait(empty + j % STAGES, (j / STAGES) & 1, d.err)) break;
          for (uint32_t j = ait > (uint32_t)Cfg::A_STAGES ? ait - Cfg::A_STAGES : 0; j < ait; j++)
            if (!mbar_wait(aempty + j % Cfg::A_STAGES, (j / Cfg::A_STAGES) & 1, d.err)) break;
        }
      }
    } else if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = t_first; t < ntiles && ok; t += t_step) {
        // PAIR: the peer's tile of a last unit with an odd tile count lies past the end: its boxes read
        // the zero fill (TMA out-of-range), its epilogue stores nothing
        const int tn_q = d.f_ntn.quo(t), nt = d.f_ntn.rem(t, tn_q), mt = PAIR ? tn_q * 2 + (int)rank : tn_q;
        const int n0 = nt * BN + (int)rank * Cfg::B_ROWS;
        int q0 = 0, p0 = 0, b0 = 0, m0 = 0;
        if (MODE == A_GEMM) {
          m0 = mt * 128;
        } else {
          const int rest = d.f_tq.quo(mt), rp = d.f_tp.quo(rest);
          q0 = d.f_tq.rem(mt, rest) * d.tw;
          p0 = d.f_tp.rem(rest, rp) * d.th;
          b0 = rp * d.tn;
        }
        for (int kb = 0; kb < d.nk; kb++, it++) {
          const int s = it % STAGES;
          if (it >= STAGES && !mbar_wait(empty + s, ((it / STAGES) - 1) & 1, d.err)) {
            ok = false;
            break;
          }
          const int tap = d.f_nkc.quo(kb), cc = d.f_nkc.rem(kb, tap) * BK;  // taps outer, channel chunks inner
          uint8_t* a = sA + s * Cfg::A_BYTES;
          uint8_t* b = sB + s * Cfg::B_BYTES;
          int ca[5] = {cc, 0, 0, 0, 0};  // A box coordinates
          if (MODE == A_GEMM) {
            ca[1] = m0;
          } else {
            const int r = d.f_S.quo(tap), c = tap - r * d.S;
            if (MODE == A_S1) {
              ca[1] = q0 + c - d.pad;
              ca[2] = p0 + r - d.pad;
              ca[3] = b0;
            } else {
              const int dr = r - d.pad, dc = c - d.pad;
              ca[0] = (dc & 1) * d.C + cc;
              ca[1] = q0 + (dc >> 1);
              ca[2] = dr & 1;
              ca[3] = p0 + (dr >> 1);
              ca[4] = b0;
            }
          }
          if (PAIR) {
            const uint32_t fb = mapa_shared(full + s, 0);  // the leader's full barrier counts both CTAs
            if (rank == 0) mbar_arrive_expect_tx(full + s, 2 * Cfg::STAGE_BYTES);
            if (MODE == A_GEMM)
              tma_load_2d_cg2(a, &ta, fb, ca[0], ca[1]);
            else if (MODE == A_S1)
              tma_load_4d_cg2(a, &ta, fb, ca[0], ca[1], ca[2], ca[3]);
            else
              tma_load_5d_cg2(a, &ta, fb, ca[0], ca[1], ca[2], ca[3], ca[4]);
            tma_load_2d_cg2(b, &tb, fb, tap * d.C + cc, n0);
          } else {
            mbar_arrive_expect_tx(full + s, Cfg::STAGE_BYTES);
            if (MODE == A_GEMM)
              tma_load_2d(a, &ta, full + s, ca[0], ca[1]);
            else if (MODE == A_S1)
              tma_load_4d(a, &ta, full + s, ca[0], ca[1], ca[2], ca[3]);
            else
              tma_load_5d(a, &ta, full + s, ca[0], ca[1], ca[2], ca[3], ca[4]);
            tma_load_2d(b, &tb, full + s, tap * d.C + cc, n0);
          }
        }
      }
      // PAIR: the leader's last commits arrive on this CTA's empty barriers; wait for them so that
      // none lands after the CTA has retired
      if (PAIR && ok) {
        for (uint32_t j = it > (uint32_t)STAGES ? it - STAGES : 0; j < it; j++)
          if (!mbar_wait(empty + j % STAGES, (j / STAGES) & 1, d.err)) break;
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if constexpr (W3) {
      if (lane == 0 && rank == 0) {
        constexpr uint32_t idesc = idesc_f16_f32(PAIR ? 256 : 128, BN);
        // row tap r starts at window pixel row r·ni·tw (stride 1) or 8·(r + 1) (stride 2, SBO 16 rows)
        const uint32_t tap_rows_bytes = (uint32_t)((S2W ? 8 : d.tn * d.tw) * Cfg::ROW_BYTES);
        const uint32_t tap_base_bytes = S2W ? 8u * Cfg::ROW_BYTES : 0u;
        constexpr uint32_t a_sbo = (S2W ? 16 : 8) * Cfg::ROW_BYTES;
        uint32_t it = 0, ait = 0, lt = 0;
        bool ok = !RESB || mbar_wait(full, 0, d.err);  // RESB: the resident weights have landed
        for (int t = t_first; t < ntiles && ok; t += t_step, lt++) {
          const uint32_t buf = lt & 1;
          if (lt >= 2) {
            const bool drained = PAIR ? mbar_wait_cluster(acce + buf, ((lt >> 1) - 1) & 1, d.err)
                                      : mbar_wait(acce + buf, ((lt >> 1) - 1) & 1, d.err);
            if (!drained) break;
          }
          tc_fence_after();
          const uint32_t dt = tmem + buf * Cfg::ACC_COLS;
          uint32_t acc = 0;
          for (int cc = 0; cc < d.C && ok; cc += BK) {
            for (int c = 0; c < 3 && ok; c++, ait++) {
              const int ws = ait % Cfg::A_STAGES;
              if (!mbar_wait(afull + ws, (ait / Cfg::A_STAGES) & 1, d.err)) {
                ok = false;
                break;
              }
              tc_fence_after();
              const uint32_t wa = smem_u32(sA + ws * Cfg::WIN_BYTES);
              for (int r = 0; r < 3; r++, it++) {
                const int s = RESB ? r * 3 + c : (int)(it % STAGES);  // RESB: the tap's resident weights
                if (!RESB && !mbar_wait(full + s, (it / STAGES) & 1, d.err)) {
                  ok = false;
                  break;
                }
                tc_fence_after();
                const uint32_t a = wa + tap_base_bytes + r * tap_rows_bytes, b = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
                for (int k = 0; k < BK / 16; k++) {
                  const uint64_t da = smem_desc_kmajor_sbo(a + k * 32, Cfg::ROW_BYTES, a_sbo);
                  const uint64_t db = smem_desc_kmajor(b + k * 32, Cfg::ROW_BYTES);
                  if (PAIR)
                    umma_f16_pair(dt, da, db, idesc, acc);
                  else
                    umma_f16(dt, da, db, idesc, acc);
                  acc = 1;
                }
                if (!RESB) {
                  if (PAIR)
                    umma_commit_pair(empty + s);
                  else
                    umma_commit(empty + s);
                }
              }
              // after the window's three taps (or what of them was issued)
              if (PAIR)
                umma_commit_pair(aempty + ws);
              else
                umma_commit(aempty + ws);
            }
          }
          if (ok) {
            if (PAIR)
              umma_commit_pair(accf + buf);
            else
              umma_commit(accf + buf);
          }
        }
      }
    } else if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = idesc_f16_f32(PAIR ? 256 : 128, BN);
      uint32_t it = 0, lt = 0;
      bool ok = true;
      for (int t = t_first; t < ntiles && ok; t += t_step, lt++) {
        const uint32_t buf = lt & 1;
        if (lt >= 2) {
          const bool drained = PAIR ? mbar_wait_cluster(acce + buf, ((lt >> 1) - 1) & 1, d.err)
                                    : mbar_wait(acce + buf, ((lt >> 1) - 1) & 1, d.err);
          if (!drained) break;
        }
        tc_fence_after();
        const uint32_t dt = tmem + buf * Cfg::ACC_COLS;
        for (int kb = 0; kb < d.nk; kb++, it++) {
          const int s = it % STAGES;
          if (!mbar_wait(full + s, (it / STAGES) & 1, d.err)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a = smem_u32(sA + s * Cfg::A_BYTES), b = smem_u32(sB + s * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) {
            const uint64_t da = smem_desc_kmajor(a + k * 32, Cfg::ROW_BYTES);
            const uint64_t db = smem_desc_kmajor(b + k * 32, Cfg::ROW_BYTES);
            if (PAIR)
              umma_f16_pair(dt, da, db, idesc, (kb | k) != 0);
            else
              umma_f16(dt, da, db, idesc, (kb | k) != 0);
          }
          if (PAIR)
            umma_commit_pair(empty + s);
          else
            umma_commit(empty + s);
        }
        if (ok) {
          if (PAIR)
            umma_commit_pair(accf + buf);
          else
            umma_commit(accf + buf);
        }
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..)
    grid_dep_wait();
    load_epilogue_consts(d.ep, d.gemm_n, 0, d.gemm_n, threadIdx.x - 64, 32 * Cfg::EPI_WARPS, s_sc, s_sh);
    named_bar_sync(1, 32 * Cfg::EPI_WARPS);
    const EpiDev& e = d.ep;
    const int ew = warp - 2;                 // 0..EPI_WARPS-1
    const int quad = warp & 3;               // TMEM lane quadrant this warp may access
    const int half = ew >> 2;                // which half of the tile's columns (8 epilogue warps)
    const int row = quad * 32 + lane;
    // 8 epilogue warps: the first half takes the leading ceil32(BN/2) columns, the second the rest, so
    // both halves are multiples of 32 for every BN % 32 == 0 (e.g. 224 → 128 + 96).
    constexpr int SPLIT = ((BN / 2 + 31) / 32) * 32;
    const int cols = Cfg::EPI_WARPS == 4 ? BN : (half == 0 ? SPLIT : BN - SPLIT);
    const int cbeg = Cfg::EPI_WARPS == 4 ? 0 : half * SPLIT;
    uint8_t* stage = s_stage + ew * (32 * 64);
    const uint32_t acce_leader = PAIR ? mapa_shared(acce, 0) : 0;  // drained barriers live in the leader
    uint32_t lt = 0;
    for (int t = t_first; t < ntiles; t += t_step, lt++) {
      const int tn_q = d.f_ntn.quo(t), nt = d.f_ntn.rem(t, tn_q), mt = PAIR ? tn_q * 2 + (int)rank : tn_q;
      const int n0 = nt * BN;
      if (PAIR && mt >= d.tiles_m) {  // the peer's tile of an odd last unit: nothing to store
        const uint32_t buf = lt & 1;
        if (!mbar_wait(accf + buf, (lt >> 1) & 1, d.err)) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(acce_leader + buf * 8);
        continue;
      }
      bool valid;
      long long pix;
      int n, p, q;
      if (MODE == A_GEMM) {
        const long long m = (long long)mt * 128 + row;
        valid = m < d.M;
        pix = m;
        q = (int)(m % d.Q);
        const long long tt = m / d.Q;
        p = (int)(tt % d.P);
        n = (int)(tt / d.P);
      } else if (W3) {  // GEMM rows in (row, image, column) order
        const int rest = d.f_tq.quo(mt), tq = d.f_tq.rem(mt, rest), rp = d.f_tp.quo(rest);
        const int i = d.f_nw.quo(row), rr = d.f_nw.rem(row, i), ni = d.f_tw.quo(rr), j = d.f_tw.rem(rr, ni);
        n = rp * d.tn + ni;
        p = d.f_tp.rem(rest, rp) * d.th + i;
        q = tq * d.tw + j;
        valid = n < d.N && p < d.P && q < d.Q;
        pix = ((long long)n * d.P + p) * d.Q + q;
      } else {
        const int rest = d.f_tq.quo(mt), tq = d.f_tq.rem(mt, rest), rp = d.f_tp.quo(rest);
        const int ni = d.f_thw.quo(row), rr = d.f_thw.rem(row, ni), i = d.f_tw.quo(rr), j = d.f_tw.rem(rr, i);
        n = rp * d.tn + ni;
        p = d.f_tp.rem(rest, rp) * d.th + i;
        q = tq * d.tw + j;
        valid = n < d.N && p < d.P && q < d.Q;
        pix = ((long long)n * d.P + p) * d.Q + q;
      }
      int bq = 0, bp = 0, bn = 0;  // origin of this warp's 32-row box (TMA-store epilogue)
      if (W3) {
        // the store maps are (C, Q, N, P) views, so their 3rd and 4th coordinates are image and row:
        // passed in the (bp, bn) slots.  A warp's 32 rows are 32 / (ni·tw) whole tile rows.
        const int rest = d.f_tq.quo(mt), rp = d.f_tp.quo(rest);
        bq = d.f_tq.rem(mt, rest) * d.tw;
        bp = rp * d.tn;
        bn = d.f_tp.rem(rest, rp) * d.th + d.f_nw.quo(quad * 32);
      } else if (MODE != A_GEMM) {
        const int rest = d.f_tq.quo(mt), rp = d.f_tp.quo(rest);
        const int w0 = quad * 32, wq = d.f_tw.quo(w0);
        bq = d.f_tq.rem(mt, rest) * d.tw + d.f_tw.rem(w0, wq);
        bp = d.f_tp.rem(rest, rp) * d.th + (wq & (d.th - 1));
        bn = rp * d.tn + d.f_thw.quo(w0);
      }
      const uint32_t buf = lt & 1;
      // the residual of the first 32 columns is loaded before the accumulator is ready; each later pass's
      // at the start of that pass, ahead of its TMEM load and math
      const bool pre_res = e.tstore && e.kind == OSAM_EPI_BN_ACT && e.res != nullptr;
      uint4 rcur[4];
      if (pre_res) residual_rows(e, valid ? pix : -1LL, d.K, n0 + cbeg, rcur);
      const bool ok = mbar_wait(accf + buf, (lt >> 1) & 1, d.err);
      tc_fence_after();
      if (!ok) break;
      const uint32_t dt = tmem + buf * Cfg::ACC_COLS + ((uint32_t)(quad * 32) << 16);
      if (e.tstore) {
#pragma unroll 1
        for (int c = 0; c < cols; c += 32) {
          __syncwarp();
          if (pre_res && c > 0) residual_rows(e, valid ? pix : -1LL, d.K, n0 + cbeg + c, rcur);
          uint32_t r0[16], r1[16];
          tmem_ld16_nowait(dt + cbeg + c, r0);
          tmem_ld16_nowait(dt + cbeg + c + 16, r1);
          tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int i = 0; i < 16; i++) {
            v[i] = __uint_as_float(r0[i]);
            v[16 + i] = __uint_as_float(r1[i]);
          }
          epilogue_warp_tma(e, sm, d.K, d.P, d.Q, v, n0 + cbeg + c, s_sc, s_sh, valid, n, p, q, bq, bp, bn, stage,
                            nullptr, pre_res ? rcur : nullptr);
        }
      } else if (e.coop) {
#pragma unroll 1
        for (int c = 0; c < cols;) {
          __syncwarp();
          const int col = n0 + cbeg + c;
          if (cols - c >= 32) {
            uint32_t r0[16], r1[16];
            tmem_ld16_nowait(dt + cbeg + c, r0);
            tmem_ld16_nowait(dt + cbeg + c + 16, r1);
            tmem_wait_ld();
            float v[32];
#pragma unroll
            for (int i = 0; i < 16; i++) {
              v[i] = __uint_as_float(r0[i]);
              v[16 + i] = __uint_as_float(r1[i]);
            }
            epilogue_warp<32>(e, d.K, d.P, d.Q, v, col, s_sc, s_sh, valid, n, p, q, stage);
            c += 32;
          } else {
            uint32_t r0[16];
            tmem_ld16_nowait(dt + cbeg + c, r0);
            tmem_wait_ld();
            float v[16];
#pragma unroll
            for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r0[i]);
            epilogue_warp<16>(e, d.K, d.P, d.Q, v, col, s_sc, s_sh, valid, n, p, q, stage);
            c += 16;
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < cols; c += 16) {
          __syncwarp();
          float v[16];
          tmem_ld16(dt + cbeg + c, v);
          const int col0 = n0 + cbeg + c;
          if (!valid || col0 >= d.gemm_n) continue;
#pragma unroll
          for (int h = 0; h < 2; h++) {
            const int col = col0 + h * 8;
            if (col >= d.gemm_n) break;
            const int cnt = d.gemm_n - col < 8 ? d.gemm_n - col : 8;
            float y[8];
#pragma unroll
            for (int i = 0; i < 8; i++) y[i] = v[h * 8 + i];
            epilogue8(e, d.K, d.P, d.Q, y, cnt, col, col, s_sc, s_sh, pix, n, p, q);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        if (PAIR)
          mbar_arrive_cluster(acce_leader + buf * 8);
        else
          mbar_arrive(acce + buf);
      }
    }
  }
  if (warp >= 2 && lane == 0) bulk_wait_group0();  // tensor stores complete before the CTA retires
  tc_fence_before();
  // PAIR: neither CTA frees its TMEM or retires while the other may still signal it
  if (PAIR) {
    __syncwarp();  // lanes 1–31 of the producer and MMA warps wait here for lane 0
    cluster_sync_all();
  } else {
    __syncthreads();
  }
  if (warp == 1) {
    tc_fence_after();
    if (PAIR)
      tmem_dealloc_pair(tmem, Cfg::TMEM_COLS);
    else
      tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
}

template <int BK, int BN, int MODE, bool PAIR>
static cudaError_t launch_one(const ConvLaunch& L, cudaStream_t st, bool prime_only) {
  using Cfg = FpropCfg<BK, BN, PAIR, MODE>;
  auto kern = k_conv_fprop<BK, BN, MODE, PAIR>;
  // The dynamic shared-memory opt-in is set once per process (one device per process) and, through
  // conv_prime(), before any stream capture.
  static bool attr_set = false;
  static int slots = 0;  // CTAs (PAIR: clusters) that run at once
  if (!attr_set) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM_BYTES);
    if (e != cudaSuccess) return e;
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
    slots = sms * Cfg::CTAS_PER_SM;
    // PAIR: one cluster per two CTA slots.  (The occupancy query for a cluster launch reports one CTA per
    // SM for the ≤ 128-wide configurations, yet two co-reside in practice: measured.  Clusters beyond
    // what fits simply wait; nothing depends on their co-residence.)
    if (PAIR) slots /= 2;
    attr_set = true;
  }
  if (prime_only) return cudaSuccess;
  // programmatic dependent launch (the kernel waits for its predecessor itself: grid_dep_wait)
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.blockDim = dim3(Cfg::THREADS);
  cfg.dynamicSmemBytes = Cfg::SMEM_BYTES;
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (!PAIR) {
    cfg.gridDim = dim3(L.grid < slots ? L.grid : slots);
  } else {
    const int units = ((L.d.tiles_m + 1) / 2) * L.d.ntn;
    at[1].id = cudaLaunchAttributeClusterDimension;
    at[1].val.clusterDim.x = 2;
    at[1].val.clusterDim.y = 1;
    at[1].val.clusterDim.z = 1;
    cfg.numAttrs = 2;
    cfg.gridDim = dim3(2 * (units < slots ? units : slots));
  }
  return cudaLaunchKernelEx(&cfg, kern, L.ta, L.tb, L.sm, L.d);
}

template <int BK, int BN>
cudaError_t launch_mode(const ConvLaunch& L, cudaStream_t st, bool prime) {
  // CTA pairs need each CTA's half of the weight rows to keep 1024-byte stages (BN/2 rows of BK)
  constexpr bool kPairOk = (BN / 2) * BK * 2 % 1024 == 0;
  if (kPairOk && L.pair) {
    switch (L.mode) {
      case A_GEMM: return launch_one<BK, BN, A_GEMM, kPairOk>(L, st, prime);
      case A_S1: return launch_one<BK, BN, A_S1, kPairOk>(L, st, prime);
      case A_S2: return launch_one<BK, BN, A_S2, kPairOk>(L, st, prime);
      case A_W3: return launch_one<BK, BN, A_W3, kPairOk>(L, st, prime);
      case A_W3R:
        if constexpr (BN == 32 || BN == 64) return launch_one<BK, BN, A_W3R, kPairOk>(L, st, prime);
        break;
      case A_W3S2:
        if constexpr (BN == 32 || BN == 64 || BN == 128) return launch_one<BK, BN, A_W3S2, kPairOk>(L, st, prime);
        break;
      case A_W3S2R:
        if constexpr (BN == 32 || BN == 64) return launch_one<BK, BN, A_W3S2R, kPairOk>(L, st, prime);
        break;
    }
    return cudaErrorInvalidValue;
  }
  switch (L.mode) {
    case A_GEMM: return launch_one<BK, BN, A_GEMM, false>(L, st, prime);
    case A_S1: return launch_one<BK, BN, A_S1, false>(L, st, prime);
    case A_S2: return launch_one<BK, BN, A_S2, false>(L, st, prime);
    case A_W3: return launch_one<BK, BN, A_W3, false>(L, st, prime);
    case A_W3R:
      if constexpr (BN == 32 || BN == 64) return launch_one<BK, BN, A_W3R, false>(L, st, prime);
      break;
    case A_W3S2:
      if constexpr (BN == 32 || BN == 64 || BN == 128) return launch_one<BK, BN, A_W3S2, false>(L, st, prime);
      break;
    case A_W3S2R:
      if constexpr (BN == 32 || BN == 64) return launch_one<BK, BN, A_W3S2R, false>(L, st, prime);
      break;
  }
  return cudaErrorInvalidValue;
}

}  // namespace osam
