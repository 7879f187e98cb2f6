"""Test infrastructure: CPU restatements of the reference's algorithms, used only as checkers.

Nothing in the product (objectsam_b200/) imports this package.  It is used by tests/, by
__graft_entry__.smoke() to check the GPU result, and by bench.py's CPU-baseline / reference arm.

  fsow.py          FSOW tensor-file reader/writer (reference src/fsow.h:28-67, pytools/fsow.py:1-44)
  yolo_params.py   YOLOv8s-seg nc=1 parameter table + seeded He-normal weight generator
                   (names/shapes of reference src/model.cpp:95-275)
  yolo_ref.py      PyTorch CPU forward of the network (reference src/model.cpp:168-275, src/bn.cu:204-238,
                   src/misc.cu:32-46), optionally emulating the reference's fp16 storage points
  postproc_ref.py  decode / greedy NMS / mask assembly (reference archive/tools/ref_detect.py:37-81,
                   DFL decode src/loss.cu:128-147)

Parity pin: the post-process restatement is checked against fixtures produced by running the
reference's own ref_detect.py (tests/golden/make_postproc_golden.py); the network restatement is
checked against fixtures produced by the reference's own cuDNN build (oracle/_ref, see oracle/Makefile).
"""
