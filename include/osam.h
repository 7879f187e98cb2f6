/* osam.h — C ABI of the ObjectSAM B200 convolution hot path.
 *
 * The reference hands every YOLOv8s-seg convolution to cuDNN through the C++ class ConvOp
 * (reference src/conv.h:16-53, src/conv.cpp) and applies BatchNorm+SiLU, bias and SPPF pooling in
 * separate passes (src/bn.cu, src/misc.cu).  This header is the plain-C boundary that replaces those
 * calls: raw device pointers and sizes, an explicit CUDA stream, int status codes, no C++ or torch
 * types.  A ConvOp-compatible C++ shim and the Python host layer sit on top of it.
 *
 * Conventions (same as the reference, src/conv.h:16-31, src/bn.cuh:9-21):
 *   - activations are NHWC packed fp16 (__half), weights are KRSC fp16 (K, R, S, C);
 *   - the transposed conv (ConvTranspose2d k=s=2) takes weights as (C_in, R, S, C_out), the layout
 *     the reference keeps for it (src/model.h:24 "layout 2");
 *   - accumulation is fp32;
 *   - every pointer handed to a kernel is 16-byte aligned and every channel count/offset used by an
 *     epilogue destination is a multiple of 8, except single-channel outputs (K = 1).
 *   - No conv, BN, pooling or post-process entry point allocates device memory, plan creation included;
 *     only osam_model_create / osam_model_train_init / osam_model_sync_weights allocate (the model's arenas).
 * All functions return OSAM_OK (0) or a positive error code; osam_last_error() describes the last one.
 */
#ifndef OSAM_H_
#define OSAM_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* osam_stream_t; /* a cudaStream_t; NULL = legacy default stream */

enum {
  OSAM_OK = 0,
  OSAM_ERR_INVALID = 1,     /* bad argument / unsupported geometry */
  OSAM_ERR_UNSUPPORTED = 2, /* valid for the reference, not implemented by this build */
  OSAM_ERR_CUDA = 3,        /* CUDA runtime/driver error */
  OSAM_ERR_TIMEOUT = 4,     /* a device-side wait ran out of its budget (kernel returned early) */
  OSAM_ERR_NOMEM = 5
};

/* Conv geometry.  Replaces ConvGeom (reference src/conv.h:8-14); P = (H+2pad-R)/stride+1. */
typedef struct osam_conv_geom {
  int N, H, W, C; /* input */
  int K, R, S;    /* output channels, kernel */
  int stride, pad;
} osam_conv_geom;

/* One output destination of a fused epilogue.  Replaces Dest (reference src/bn.cuh:10-17):
 * output channels [c0, c1) go to channels [choff, choff + c1 - c0) of an NHWC buffer with ctot
 * channels; up = 2 writes each pixel to its 2×2 nearest-neighbour block of a 2P×2Q buffer. */
typedef struct osam_dest {
  void* p;
  int ctot, choff, c0, c1, up;
} osam_dest;

#define OSAM_MAX_DEST 4

enum {
  OSAM_EPI_STORE = 0,  /* y = conv (+ beta·y): the plain ConvOp::fwd contract */
  OSAM_EPI_BN_ACT = 1, /* a = act(scale·z + shift) (+ res) → dests: conv + bn_forward_apply (src/bn.cu:204-238) */
  OSAM_EPI_BIAS = 2    /* y = z + bias → dests: conv + add_bias (src/misc.cu:116-134, src/model.cpp:403-407) */
};

/* Fused epilogue of a forward conv (the folded-BN / bias / residual / DestList store). */
typedef struct osam_epilogue {
  int kind;             /* OSAM_EPI_* */
  const float* scale;   /* [K] BN_ACT: γ/√(var+eps) */
  const float* shift;   /* [K] BN_ACT: β − μ·scale   (bn_eval_scale, src/bn.cu:277-284) */
  const float* bias;    /* [K] BIAS */
  const void* res;      /* BN_ACT: optional residual [N,P,Q,K] fp16 added after the activation */
  int act;              /* BN_ACT: 1 = SiLU */
  int round_z;          /* 1: round the fp32 accumulator to fp16 before the epilogue math, as the
                           reference does by storing z in fp16 (src/model.cpp:388-400) */
  int n_dest;
  osam_dest dest[OSAM_MAX_DEST];
} osam_epilogue;

typedef struct osam_conv_plan osam_conv_plan;

/* Plan for one conv geometry.  Replaces ConvOp::init + tune (src/conv.h:21-27): tile shapes are a
 * static function of the geometry, so there is nothing to time.  transposed = 1 means
 * ConvTranspose2d(C→K, kernel R=S=stride, pad 0) as in ConvOp::init(…, transposed=true). */
int osam_conv_plan_create(const osam_conv_geom* g, int transposed, osam_conv_plan** out);
int osam_conv_plan_destroy(osam_conv_plan* plan);
/* Workspace bytes the caller must pass to fwd/dgrad/wgrad (ConvOp::tune's return value). */
size_t osam_conv_workspace_size(const osam_conv_plan* plan);
/* Output elements N·P·Q·K (ConvOp::out_elems, src/conv.h:33). */
int64_t osam_conv_out_elems(const osam_conv_plan* plan);

/* y = conv(x, w) (+ beta·y).  Replaces ConvOp::fwd (src/conv.h:29, src/conv.cpp:335-344). */
int osam_conv_fwd(const osam_conv_plan* plan, const void* x, const void* w, void* y, float beta, void* ws,
                  size_t ws_bytes, osam_stream_t stream);

/* dx = dgrad(dz, w) (+ beta·dx): the input gradient of the plan's forward conv, dz N×P×Q×K → dx N×H×W×C,
 * beta 0 (overwrite) or 1 (accumulate, the reference's dgrad_accum).  Replaces ConvOp::dgrad (src/conv.h:30,
 * src/conv.cpp:346-355).  Runs on the forward kernels over dz with re-laid-out weights written to the
 * workspace (osam_conv_workspace_size, 256-byte aligned): one conv for stride 1, one per output-parity
 * class for stride 2.  Transposed plans (kernel = stride = 2, src/conv.cpp:351-353): dx is the stride-2 2×2
 * conv of dy with the transposed conv's own (C_in, R, S, C_out) weights read as KRSC; no workspace.
 * OSAM_ERR_UNSUPPORTED for non-square kernels or output channels that the forward kernels cannot take as
 * inputs (not a multiple of 32). */
int osam_conv_dgrad(const osam_conv_plan* plan, const void* dz, const void* w, void* dx, float beta, void* ws,
                    size_t ws_bytes, osam_stream_t stream);

/* dw = wgrad(x, dz) (+ beta·dw): the weight gradient of the plan's forward conv, x N×H×W×C and
 * dz N×P×Q×K → dw K×R×S×C fp16 (KRSC, like the reference's gw_act).  Replaces ConvOp::wgrad (src/conv.h:31,
 * src/conv.cpp:357-366).  Accumulates in fp32 in the workspace (osam_conv_workspace_size, 256-byte
 * aligned), which it zeroes itself.  Small-C plans (R·S·C ≤ 32, the RGB stem) take K = 32 or 64 and replace
 * the reference's wgrad_rgb_s2 (src/misc.cu:193-273, src/model.cpp:421-422) for any size and stride.
 * Transposed plans (src/conv.cpp:362-364): dw[c][r][s][k] = Σ x[p][q][c]·dy[2p+r][2q+s][k] in the
 * (C_in, R, S, C_out) layout, run as the weight gradient of that stride-2 conv.
 * OSAM_ERR_UNSUPPORTED for other channel counts that are not multiples of 32. */
int osam_conv_wgrad(const osam_conv_plan* plan, const void* x, const void* dz, void* dw, float beta, void* ws,
                    size_t ws_bytes, osam_stream_t stream);

/* Conv fused with its epilogue (BN fold + SiLU + residual + multi-destination store, or bias).
 * Replaces ConvOp::fwd followed by bn_eval_scale/bn_forward_apply (src/model.cpp:388-400) or by
 * add_bias (src/model.cpp:405-406). */
int osam_conv_fwd_fused(const osam_conv_plan* plan, const void* x, const void* w, const osam_epilogue* ep,
                        void* ws, size_t ws_bytes, osam_stream_t stream);

/* Transposed-conv forward that allocates nothing and takes no workspace: same result as
 * osam_conv_fwd on a transposed plan, but the weights' re-laid-out copy goes to a fixed device array
 * inside the library instead of a caller-provided workspace.  It has no counterpart in the reference
 * (its ConvOp always receives a workspace from the caller).  It is meant for callers that cannot
 * allocate device memory or hand out a workspace: a host that owns the whole device budget and gives
 * a plugin only a stream, or a loop that must never reach the allocator because cudaMalloc can
 * synchronise the device.
 * Limit: C_in · 4 · C_out fp16 weights ≤ 256 KiB (C_in · C_out ≤ 32768, e.g. 128 → 128); larger plans
 * return OSAM_ERR_INVALID.  Every GPU that loads the library holds the 256 KiB array until exit.
 * The array is shared by all calls on a device and keeps the last call's contents: calls that overlap
 * on the GPU (e.g. on two streams) race on it.  The first call on each device looks the array's device
 * address up (cudaGetSymbolAddress) with that device current; make that first call before any stream
 * capture begins.  Needs a transposed plan (OSAM_ERR_INVALID otherwise). */
int osam_convt_fwd_static_scratch(const osam_conv_plan* plan, const void* x, const void* w, void* y, float beta,
                                  osam_stream_t stream);

/* SPPF pooling: with cv1's output in channels [0,c) of cat (N×H×W×4c), writes the three chained
 * 5×5/s1/p2 max-pools into slices 1..3.  Replaces sppf_pool_fwd (src/misc.cuh:6, src/misc.cu:149-153). */
int osam_sppf_fwd(void* cat, int N, int H, int W, int c, osam_stream_t stream);

/* SPPF backward: with the forward's cat (N×H×W×4c, slices 0..3) and the gradients of all four slices in
 * dcat, routes slice 3's gradient back through the three chained pools (each output position to the first
 * maximum of its clipped 5×5 window, row-major, as PyTorch) and ADDS the result to dcat slice 0; slices 1–3
 * of dcat are left as they are.  Needs no workspace (the reference's two fp32 scratch buffers stay on chip).
 * Replaces sppf_pool_bwd (src/misc.cuh:9-10, src/misc.cu:48-73, :155-166).  c % 8 == 0;
 * OSAM_ERR_UNSUPPORTED when H·W > 1816 (the per-CTA shared memory). */
int osam_sppf_bwd(const void* cat, void* dcat, int N, int H, int W, int c, osam_stream_t stream);

/* ------------------------------------------------------------------------------------------------
 * Training-mode BatchNorm + SiLU and the head-conv bias passes (the reference's src/bn.cuh:23-47 and
 * src/misc.cuh:13-17).  z, residuals and gradients are NHWC fp16 [N·H·W][C] with C a multiple of 8,
 * C ≤ 2048; per-channel vectors are fp32.  Statistics reduce in fp32 per thread and CTA, then fp64.
 * Workspaces: osam_bn_workspace_size(C) / osam_chan_sum_workspace_size(C) bytes, 16-byte aligned, ZERO-FILLED
 * ONCE before first use (the reference's bn_init, src/bn.cuh:28); every call leaves its accumulators zeroed
 * again (osam_bn_backward keeps its per-channel means in the scratch behind them, rewritten each call).  One
 * workspace serves calls issued in order on one stream; calls that may overlap need their own.
 * ------------------------------------------------------------------------------------------------ */
size_t osam_bn_workspace_size(int C);

/* scale = γ/√(running_var + eps), shift = β − running_mean·scale.  Replaces bn_eval_scale (src/bn.cuh:36,
 * src/bn.cu:277-284, :306-309). */
int osam_bn_eval_scale(int C, const float* gamma, const float* beta, const float* run_mean, const float* run_var,
                       float eps, float* scale, float* shift, osam_stream_t stream);

/* Batch statistics of z: mean, istd = 1/√(var + eps) (biased var), scale = γ·istd, shift = β − mean·scale;
 * with momentum > 0 also running_mean ← (1−m)·running_mean + m·mean and running_var ← (1−m)·running_var +
 * m·var·M/(M−1).  Needs M = N·H·W ≥ 2.  Replaces bn_forward_stats (src/bn.cuh:30-34, src/bn.cu:311-322). */
int osam_bn_forward_stats(const void* z, int N, int H, int W, int C, const float* gamma, const float* beta,
                          float* run_mean, float* run_var, float momentum, float eps, float* mean, float* istd,
                          float* scale, float* shift, void* ws, size_t ws_bytes, osam_stream_t stream);

/* a = act(scale·z + shift) (+ res, [N·H·W][C]) → 1..4 destinations (c1 = 0 means C; channel offsets and
 * ctot multiples of 8, buffers 16-byte aligned).  act = 1 is SiLU.  Replaces bn_forward_apply
 * (src/bn.cuh:42-44, src/bn.cu:204-238, :324-327). */
int osam_bn_forward_apply(const void* z, int N, int H, int W, int C, const float* scale, const float* shift,
                          const void* res, const osam_dest* dests, int n_dest, int act, osam_stream_t stream);

/* osam_bn_forward_stats followed by osam_bn_forward_apply with that scale/shift, in one call (the pair the
 * reference's forward(true) runs for every conv, src/model.cpp:389-400).  Same outputs, arguments and
 * workspace as the two calls. */
int osam_bn_forward_train(const void* z, int N, int H, int W, int C, const float* gamma, const float* beta,
                          float* run_mean, float* run_var, float momentum, float eps, float* mean, float* istd,
                          float* scale, float* shift, const void* res, const osam_dest* dests, int n_dest, int act,
                          void* ws, size_t ws_bytes, osam_stream_t stream);

/* Backward of osam_bn_forward_apply ∘ stats.  grad_dests[i].p is the GRADIENT buffer of forward
 * destination i (same ctot/choff/c0/c1/up); dA = their sum (2×2 sum for up = 2).  g = dA·silu'(y) (act),
 * dβ = Σg, dγ = Σg·x̂ into gw_beta/gw_gamma (accum ? += : =), dz = scale·(g − Σg/M − x̂·Σg·x̂/M), and with
 * res_grad non-null res_grad (res_accum ? += : =) dA.  Two passes: the sums, then dz.  Replaces bn_backward
 * (src/bn.cuh:46-50, src/bn.cu:240-270, :329-344); its `sums` scratch lives in the workspace. */
int osam_bn_backward(const void* z, int N, int H, int W, int C, const float* mean, const float* istd,
                     const float* scale, const float* shift, const osam_dest* grad_dests, int n_dest, int act,
                     void* dz, float* gw_gamma, float* gw_beta, int accum, void* res_grad, int res_accum, void* ws,
                     size_t ws_bytes, osam_stream_t stream);

/* out[c] (accum ? += : =) Σ_rows x[row][c] for x [M][C] fp16, any C ≤ 2048 (the bias gradient of the head
 * convs).  Replaces chan_sum (src/misc.cuh:13-14, src/misc.cu:103-113, :168-172). */
size_t osam_chan_sum_workspace_size(int C);
int osam_chan_sum(const void* x, int64_t M, int C, float* out, int accum, void* ws, size_t ws_bytes,
                  osam_stream_t stream);

/* y[row][c] += bias[c] for y [M][C] fp16 (one fp16 rounding of the fp32 sum).  Replaces add_bias
 * (src/misc.cuh:17, src/misc.cu:116-134, :174-177); the inference path fuses it into the conv epilogue. */
int osam_add_bias(void* y, int64_t M, int C, const float* bias, osam_stream_t stream);

/* ------------------------------------------------------------------------------------------------
 * Training mask loss of the segment head (the mask part of SegLoss::run, src/loss.cuh:53-64,
 * src/loss.cu:393-543, :613-619).  Inputs follow the reference's MaskArgs (src/loss.cu:393-408):
 *   coef[l]    NHWC fp16 [batch][h_l][w_l][32] coefficient heads, level_hw = {h0, w0, h1, w1, h2, w2}
 *              (anchors A = Σ h_l·w_l, level-major, row-major);
 *   proto      NHWC fp16 [batch][proto_h][proto_w][32] (proto_w % 16 == 0, proto_h % 8 == 0);
 *   npos[b], pos[b][A] (positive anchor ids of image b, first npos[b] entries), agt[b][A] (assigned gt of each
 *   anchor), gt_box [batch][max_gt][4] xyxy input pixels, gt_mask [batch][max_gt][proto_h·proto_w/32] bits;
 *   fg, scale: device floats (positive count of the batch, loss scale).
 * For every positive i of image b and proto pixel p in its box scaled to the proto grid:
 *   z = coef_i·proto_p, y = mask bit, loss_sum += bce(z, y)/(Hp·Wp·area_i)   (area normalised to the image)
 *   g = (σ(z) − y)·box_gain·batch/max(fg,1)·scale/(Hp·Wp·area_i),  dproto_p += g·coef_i,  dcoef_i += g·proto_p.
 * dproto is written for every pixel (zero outside all boxes); dcoef rows are written for the positive
 * anchors only (the reference's detection-loss pass zeroes the others); *loss_sum is added to.
 * Workspace: osam_mask_loss_workspace_size(batch, A) bytes, 256-byte aligned, ZERO-FILLED ONCE before first
 * use; every call leaves it zeroed again. */
size_t osam_mask_loss_workspace_size(int batch, int anchors);
int osam_mask_loss(const void* const* coef, const int* level_hw, const void* proto, int batch, int proto_h, int proto_w,
                   int imgsz, int max_gt, const int* npos, const int* pos, const int* agt, const float* gt_box,
                   const uint32_t* gt_mask, const float* fg, const float* scale, float box_gain, void* dproto,
                   void* const* dcoef, float* loss_sum, void* ws, size_t ws_bytes, osam_stream_t stream);

/* ------------------------------------------------------------------------------------------------
 * Detection part of the training loss (SegLoss::run before its mask part: src/loss.cuh:53-64,
 * src/loss.cu:123-390, :590-612; Ultralytics 8.4 v8SegmentationLoss, one class, reg_max 16, top-10 TAL).
 *   box[l] / cls[l]: NHWC fp16 heads [batch][h_l][w_l][64] / [..][1], level_hw = {h0, w0, h1, w1, h2, w2};
 *   n_gt[batch], gt_box [batch][max_gt][4] xyxy input pixels, ignore [batch][proto_h·proto_w/32] bits or NULL
 *   (a negative anchor whose centre lies in it gets no class loss); scale: device float (gradients only).
 * DFL decode → per gt the 10 in-box anchors (box enlarged to ≥ 16 px) of highest √score·CIoU⁶ (ties: lower
 * anchor) → per anchor its gt (most overlap when several chose it) → target scores → BCE on every anchor,
 * CIoU and DFL on the positives, with their gradients.  Writes dbox[l] and dcls[l] for every anchor, zeroes
 * the dcoef[l] rows of negatives (osam_mask_loss writes the positives'), agt [batch][A] (−1: negative), tsc
 * [batch][A] target scores, npos[batch] and pos [batch][A] (positives in anchor order), items[16]: [4]
 * positives, [5] target-score sum, [8] Σ (1 − CIoU)·t, [10] Σ BCE, [11] Σ DFL·t (the reference's layout; [9]
 * is the mask loss's: pass items + 9 as its loss_sum and items + 4 as its fg).  Workspace
 * osam_det_loss_workspace_size(batch, A, max_gt) bytes, 256-byte aligned, any contents (the call zeroes the
 * part it accumulates into). */
size_t osam_det_loss_workspace_size(int batch, int anchors, int max_gt);
int osam_det_loss(const void* const* box, const void* const* cls, const int* level_hw, int batch, int imgsz,
                  int reg_max, const int* n_gt, const float* gt_box, int max_gt, const uint32_t* ignore, int proto_h,
                  int proto_w, const float* scale, float box_gain, float cls_gain, float dfl_gain, void* const* dbox,
                  void* const* dcls, void* const* dcoef, int* agt, float* tsc, int* npos, int* pos, float* items,
                  void* ws, size_t ws_bytes, osam_stream_t stream);
/* items[0..3] = [box, seg, cls, dfl] from the sums (the reference's k_final): box = items[8]/T·box_gain,
 * seg = items[9]/fg·box_gain (0 without positives), cls = items[10]/T·cls_gain, dfl = items[11]/T·dfl_gain,
 * T = max(items[5], 1), fg = items[4]. */
int osam_seg_loss_items(float* items, float box_gain, float cls_gain, float dfl_gain, osam_stream_t stream);

/* ------------------------------------------------------------------------------------------------
 * Inference post-process (the reference has it only in numpy: archive/tools/ref_detect.py:37-81).
 * level_hw = {h0, w0, h1, w1, h2, w2} of the three head levels; anchors = Σ h·w, level-major, row-major.
 * ------------------------------------------------------------------------------------------------ */

/* DFL decode of the raw heads (NHWC fp16: box[l] 4·reg_max channels, cls[l] 1 channel) into xyxy boxes in
 * input pixels (float [batch][anchors][4]) and conf = sigmoid(cls) (float [batch][anchors]).  Follows the
 * reference's DFL decode (src/loss.cu:128-147) and the exported xywh → ref_detect xyxy conversion
 * (archive/tools/ref_detect.py:44-45). */
int osam_decode(const void* const* box, const void* const* cls, const int* level_hw, int batch, int imgsz,
                int reg_max, float* xyxy, float* conf, osam_stream_t stream);

/* Score threshold, stable descending sort and greedy NMS per image (archive/tools/ref_detect.py:41-60):
 * conf > conf_th, strict IoU > iou_th suppression (only when the union is > 0), at most max_det kept.
 * forced = 1 skips threshold and suppression and keeps the max_det highest scores.  Outputs per image:
 * n_det[b], keep[b][max_det] (anchor indices in score order, −1 padded), det_box[b][max_det][4],
 * det_score[b][max_det].  With coef (NHWC fp16 heads, 32 ch) and coef_g non-NULL, the kept anchors'
 * mask coefficients are gathered into coef_g [batch][ceil128(max_det)][32] fp16 for osam_mask_assemble.
 * Kept indices are bit-exact with the reference's loop for the same boxes and scores. */
int osam_nms(const float* xyxy, const float* conf, int batch, int anchors, float conf_th, float iou_th, int max_det,
             int forced, const void* const* coef, const int* level_hw, int* n_det, int* keep, float* det_box,
             float* det_score, void* coef_g, osam_stream_t stream);

/* Mask assembly (archive/tools/ref_detect.py:62-71) as a tensor-core GEMM per image:
 * logits = coef_g[b] (ceil128(max_det) × 32) · proto[b] (32 × Hp·Wp, proto NHWC fp16), fused with
 * mask = logit > 0 (≡ sigmoid > 0.5) ∩ the detection box scaled to the proto grid (g = Wp / imgsz).
 * masks: packed = 0 → u8 [batch][max_det][Hp·Wp]; packed = 1 → u32 [batch][max_det][ceil(Hp·Wp/32)] with
 * pixel 32·j + k in bit k of word j.  Rows ≥ n_det[b] are zero. */
int osam_mask_assemble(const void* coef_g, const void* proto, const float* det_box, const int* n_det, int batch,
                       int proto_h, int proto_w, int imgsz, int max_det, int packed, void* masks,
                       osam_stream_t stream);

/* ------------------------------------------------------------------------------------------------
 * YOLOv8s-seg (nc = 1) inference graph on the kernels above.  Replaces the reference's Model
 * (src/model.h:97-140): build (src/model.cpp:168-347), Params::load + sync_weights (:49-62, :369),
 * forward(false) (:383-414), input()/head()/proto() accessors.  Every conv node runs as one fused
 * kernel (conv + folded eval-mode BN + SiLU + residual + concat/upsample routing, or conv + bias).
 * ------------------------------------------------------------------------------------------------ */
typedef struct osam_model osam_model;

/* A device tensor owned by the model: NHWC fp16, p = base of an (n, h, w, c) buffer. */
typedef struct osam_tensor {
  void* p;
  int n, h, w, c;
} osam_tensor;

/* Build the graph and allocate all activations for `batch` images of imgsz×imgsz (imgsz % 32 == 0).
 * reg_max: DFL bins of the box head (16 for YOLOv8s-seg).  Allocates device memory (setup time). */
int osam_model_create(int batch, int imgsz, int reg_max, osam_model** out);
int osam_model_destroy(osam_model* m);
/* One parameter, PyTorch name and layout (e.g. "model.0.conv.weight" K×C×R×S), host fp32 — the
 * reference's Params::load contract.  Unknown names are ignored (returns OSAM_OK), wrong shapes fail. */
int osam_model_set_param(osam_model* m, const char* name, const float* data, const int64_t* shape, int ndim);
/* Read every parameter from an FSOW file (reference src/fsow.h format). */
int osam_model_load_fsow(osam_model* m, const char* path);
/* Upload the parameters: fp16 KRSC weights and folded eval-mode BN (γ/√(var+eps), β−μ·scale), then
 * encode every kernel's tensor maps.  All parameters must have been set. */
int osam_model_sync_weights(osam_model* m, osam_stream_t stream);
int osam_model_input(const osam_model* m, osam_tensor* t);                   /* NHWC fp16, C = 3 */
int osam_model_head(const osam_model* m, int kind, int level, osam_tensor* t); /* kind 0 box, 1 cls, 2 coef */
int osam_model_proto(const osam_model* m, osam_tensor* t);
int osam_model_act(const osam_model* m, const char* name, osam_tensor* t);   /* any named activation */
/* Inference forward pass: input → heads + proto.  use_graph = 1 records the launch sequence as a CUDA
 * graph on the first call and replays it afterwards (the first call must not be inside a capture).
 * Independent nodes run on the model's own streams forked from `stream` and joined back into it: work
 * queued on `stream` after the call sees the whole forward complete.  The first call creates those
 * streams and events. */
int osam_model_forward(osam_model* m, int use_graph, osam_stream_t stream);
/* Kernels launched by one forward pass (one per graph node). */
int osam_model_num_launches(const osam_model* m);

/* The whole inference step of BASELINE config 2 in one graph: the forward, then DFL decode, score threshold +
 * greedy NMS and the mask assembly (osam_decode / osam_nms / osam_mask_assemble) on the model's own output
 * buffers.  The post-process launches join the forward's dependency graph: decode and NMS need only the box,
 * class and coefficient heads, so they run while the proto branch is still computing; the masks wait for
 * proto.  Replaces the reference's Model::forward(false) followed by archive/tools/ref_detect.py's numpy
 * steps (:37-81).  osam_model_detect_init fixes the settings and allocates the outputs (once; again only
 * when max_det or packed change); osam_model_forward_detect runs the step (use_graph: as a captured CUDA
 * graph, recorded at the first call); osam_model_detections returns the output buffers. */
typedef struct osam_detections {
  int batch, anchors, max_det, packed, proto_h, proto_w;
  float* xyxy;    /* [batch][anchors][4] decoded boxes, input pixels */
  float* conf;    /* [batch][anchors] sigmoid(class logit) */
  int* n_det;     /* [batch] */
  int* keep;      /* [batch][max_det] kept anchors in score order, −1 padded */
  float* box;     /* [batch][max_det][4] */
  float* score;   /* [batch][max_det] */
  void* coef_g;   /* [batch][ceil128(max_det)][32] fp16 mask coefficients of the kept anchors */
  void* masks;    /* packed: u32 [batch][max_det][ceil(Hp·Wp/32)]; else u8 [batch][max_det][Hp·Wp] */
} osam_detections;
int osam_model_detect_init(osam_model* m, float conf_th, float iou_th, int max_det, int forced, int packed);
int osam_model_forward_detect(osam_model* m, int use_graph, osam_stream_t stream);
int osam_model_detections(const osam_model* m, osam_detections* d);
/* Launch nodes [first, first+count) of the forward pass on `stream` (eager), e.g. to bracket one
 * kernel with timing events.  Running every node in order equals osam_model_forward(m, 0, stream). */
int osam_model_forward_nodes(osam_model* m, int first, int count, osam_stream_t stream);
/* Geometry of node i: name (NUL-terminated, truncated to name_len), kind (0 conv+BN+SiLU, 1 head conv +
 * bias, 2 transposed conv + bias, 3 SPPF pool) and the conv geometry (pool: N,H,W,C of the slice). */
int osam_model_node_info(const osam_model* m, int i, char* name, int name_len, int* kind, osam_conv_geom* g);

/* ---- training (the reference's Model::forward(true) / Model::backward, src/model.cpp:383-470) ----
 * osam_model_train_init allocates the activation gradients, the per-node z buffers and BN state, and the fp32
 * parameter-gradient arena; it takes γ, β and the running statistics from the parameters last synced.
 * osam_model_forward_train: conv → z (fp16), batch statistics (running statistics updated with `momentum`),
 * BN + SiLU (+ residual) → destinations; the heads and proto come out as in inference.
 * The caller then writes the gradients of the heads and of proto (osam_model_act_grad on "out.box<l>",
 * "out.cls<l>", "out.coef<l>", "out.proto") and runs osam_model_backward_nodes over [first, first + count)
 * in DECREASING node order; osam_model_backward_nodes(m, 0, osam_model_num_launches(m), s) is the whole
 * backward.  Per node: BN backward (dz, dγ, dβ, residual gradient), weight gradient, input gradient
 * (accumulated where an activation feeds several nodes); heads and the transposed conv: bias gradient,
 * weight gradient, input gradient; SPPF: its backward.  Parameter gradients (fp32) sit in one arena with
 * the nodes in REVERSE order, so the gradients of nodes [first, n) are one contiguous range that a
 * data-parallel all-reduce can send while nodes before `first` are still computing.  They are written,
 * not accumulated. */
int osam_model_train_init(osam_model* m, osam_stream_t stream);
int osam_model_forward_train(osam_model* m, float momentum, osam_stream_t stream);
int osam_model_backward_nodes(osam_model* m, int first, int count, osam_stream_t stream);
int osam_model_act_grad(const osam_model* m, const char* name, osam_tensor* t); /* gradient of an activation */
int osam_model_grad_arena(const osam_model* m, float** p, int64_t* n);        /* fp32 parameter gradients */
int osam_model_node_grad_range(const osam_model* m, int i, int64_t* off, int64_t* n); /* node i's slice */
/* One parameter's gradient in its PyTorch name and layout (host fp32, n ≥ its element count); synchronous. */
int osam_model_get_grad(osam_model* m, const char* name, float* out, int64_t n);

/* ---- data-parallel training: the gradient exchange (SURVEY's multi-GPU plan for the reference's
 * src/train.cpp:209-232 step; the reference itself trains on one GPU).  One process per GPU holds a model
 * after osam_model_train_init; osam_dp_backward runs the model's whole backward in buckets of about
 * bucket_bytes of fp32 gradients (last node first) and all-reduces each bucket's gradients (ncclAvg: the sum
 * over ranks ÷ world) on a communication stream while the earlier nodes' backward continues; the caller's
 * stream waits for the exchange at the end, so an optimizer step enqueued after it reads averaged gradients
 * (the order src/optim.cu:170-175 needs).  NCCL is loaded at run time (the libnccl.so.2 already in the
 * process, else the system one).
 *   osam_dp_unique_id   rank 0 makes a communicator id (NCCL's 128-byte unique id); every rank needs it
 *   osam_dp_create      a new NON-BLOCKING communicator (world, rank, id); init_timeout_ms bounds the wait
 *                       for the other ranks (OSAM_ERR_TIMEOUT).  world = 1: no communicator, the backward
 *                       runs unbucketed-equivalent and nothing is exchanged.
 *   osam_dp_create_from_comm  over the caller's ncclComm_t (not destroyed by osam_dp_destroy)
 *   osam_dp_wait        host guard after a step: polls the exchange's completion and ncclCommGetAsyncError;
 *                       on an NCCL error, or when timeout_ms passes first (a peer died or stopped), aborts
 *                       the communicator (ncclCommAbort) and returns an error instead of hanging.
 * No counterpart in the reference. */
typedef struct osam_dp osam_dp;
int osam_dp_unique_id(unsigned char id[128]);
int osam_dp_create(osam_model* m, int world, int rank, const unsigned char id[128], size_t bucket_bytes,
                   int init_timeout_ms, osam_dp** out);
int osam_dp_create_from_comm(osam_model* m, void* nccl_comm, size_t bucket_bytes, osam_dp** out);
int osam_dp_num_buckets(const osam_dp* dp);
int osam_dp_bucket(const osam_dp* dp, int i, int* first, int* count, int64_t* off, int64_t* n);
int osam_dp_backward(osam_dp* dp, osam_stream_t stream);
int osam_dp_wait(osam_dp* dp, int timeout_ms);
int osam_dp_destroy(osam_dp* dp);

/* Device error word shared by all kernels of this library on the current device: returns the first
 * error code recorded by a kernel since the last call (0 if none) and clears it.  Synchronises.
 * Launches are asynchronous, so a kernel whose bounded wait ran out (OSAM_ERR_TIMEOUT: it returned early
 * and its output is incomplete) is seen here, not in the status of the call that launched it; callers
 * check it at a point where they synchronise anyway, or poll osam_device_error_peek.  The word is one int
 * of host-mapped pinned memory allocated at the first plan or model creation (a static device variable
 * before that); no launch allocates.  No counterpart in the reference (cuDNN has no device-side status;
 * its kernels cannot time out). */
int osam_device_error(void);

/* The error word as it stands, read from host-mapped memory without synchronising anything and without
 * clearing it: non-zero once a kernel that has already finished recorded a failure.  Cheap enough to call
 * before every launch (the ConvOp shim does, and aborts like the reference's FSO_ASSERT).  Covers kernels
 * launched after the first plan or model creation, which allocates the mapped word (pinned host memory,
 * once per process); returns 0 before that.  No counterpart in the reference. */
int osam_device_error_peek(void);

/* Self-test of the bounded device waits: launches one thread that waits on an mbarrier nothing arrives
 * at, with a budget of budget_ns (at most 5 s); the wait runs out, records OSAM_ERR_TIMEOUT in the device
 * error word and the kernel returns, leaving the context usable.  For tests; no counterpart in the
 * reference. */
int osam_selftest_wait_timeout(unsigned long long budget_ns, osam_stream_t stream);

/* ---- training-batch augmentation (reference src/augment.cuh:19 `augment`, kernels src/augment.cu) ----
 * The loader's batch description, field for field the reference's (src/dataset.h:19-47): its loader fills
 * these structs on the host and copies them to the device unchanged, so the layouts must agree. */
typedef struct osam_aug_src {   /* ≙ SrcInfo: one source image */
  int64_t img_off;              /* byte offset of its RGB u8 pixels (rows of iw·3) in the image block */
  int iw, ih;                   /* image size */
  int mw, mh;                   /* instance-mask resolution */
} osam_aug_src;
typedef struct osam_aug_inst {  /* ≙ InstInfo: one instance, in source-image coordinates */
  int src;                      /* osam_aug_src index */
  int sample;                   /* output image */
  int tile;                     /* mosaic tile 0..3 */
  float box[4];                 /* xyxy, source pixels */
  int mx0, my0, mcw, mch;       /* its mask window (mask pixels): origin and size */
  int wpr;                      /* u32 words per mask-bitmap row */
  int64_t mask_off;             /* u32 offset of its bitmap in the mask block */
  int ignore;                   /* 1 = an ignore region (excluded from the loss), not a target */
} osam_aug_inst;
typedef struct osam_aug_sample {  /* ≙ SampleInfo: one output image */
  int src[4];                     /* source of each tile (−1: none) */
  int ta[4][4];                   /* tile rectangle on the 2S × 2S canvas: x1, y1, x2, y2 */
  int tb[4][2];                   /* where the tile starts in its source: x, y */
  float s, tx, ty;                /* canvas → output: out = s·u + t */
  float hsv[3];                   /* hue, saturation, value gains */
  int flip;                       /* mirror left-right */
  int inst0, ninst;               /* carried, not read (instances are matched by their `sample`) */
} osam_aug_sample;
typedef struct osam_aug_header {  /* ≙ BatchHeader */
  int B, S;
  int nsrc, ninst;
  int64_t img_bytes, mask_words;
} osam_aug_header;
/* Device pointers of one batch (≙ the device BatchBuf): hdr → smp[B] → src[4B] → inst[...] may be one
 * block, as the reference lays them out, or separate arrays. */
typedef struct osam_aug_batch {
  const osam_aug_header* hdr;  /* reads hdr->ninst */
  const osam_aug_sample* smp;
  const osam_aug_src* src;
  const osam_aug_inst* inst;
  const uint8_t* img;
  const uint32_t* mask;
} osam_aug_batch;
/* Outputs (≙ AugOut + GtBatch, src/augment.cuh:11-17, src/loss.cuh:25-30). */
typedef struct osam_aug_out {
  void* img;          /* fp16 [B][S][S][3] NHWC in 0..1: the model input */
  int* n_gt;          /* [B] */
  float* box;         /* [B][G][4] xyxy output pixels */
  uint32_t* mask;     /* [B][G][Hp·Wp/32] bits, cell r·Wp + c in bit (r·Wp + c) % 32 of word (r·Wp + c) / 32 */
  uint32_t* ignore;   /* [B][Hp·Wp/32] or NULL */
  int* gt_inst;       /* [B][G] instance index of each target */
  int G, Hp, Wp;      /* Wp % 32 == 0 */
} osam_aug_out;

/* ≙ augment(dev, B, S, out, stream) (src/augment.cuh:19): mosaic canvas (2S × 2S, fill 114) → affine
 * (scale + translate, bilinear) → HSV gains → left-right flip → fp16 image; targets (boxes clipped to their
 * tile, mapped, clipped to the image, flipped, kept when w, h > 2 px, area ratio > 0.1 and aspect < 100, in
 * instance order, at most G per image), their mask bits on the Hp × Wp grid and the ignore bits.  Every
 * output word is written, so the outputs need no prior zeroing.  A mask cell is S / Wp output pixels wide.
 * Requires S % 8 == 0 (S ≤ 16384), Wp % 32 == 0, G ≥ 1, hdr / src / inst 8-byte and smp 4-byte aligned (in the
 * reference's one-block layout: an even B) — OSAM_ERR_INVALID otherwise.  Pixel values, boxes and bits
 * follow the reference kernels' float steps in their order, under the same fast-math arithmetic. */
int osam_augment(const osam_aug_batch* batch, int B, int S, const osam_aug_out* out, osam_stream_t stream);

/* Human-readable description of the last error returned on this host thread. */
const char* osam_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* OSAM_H_ */
