"""Generates tests/golden/augment_golden.npz: the reference's own augmentation kernels (src/augment.cu, built
into oracle/_ref/ref_bn by oracle/Makefile, op 6) run on a seeded synthetic batch (tests/aug_batch.py,
seed 11, B 2, S 96, G 8, Hp = Wp = 32).  Needs a GPU; tests/test_augment_cpu.py rebuilds the same batch
from the seed and checks the CPU restatement oracle/augment_ref.py against these outputs.

    python tests/golden/make_augment_golden.py [out.npz]
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path[:0] = [ROOT, os.path.dirname(HERE)]

from aug_batch import make_batch  # noqa: E402
from test_augment_gpu import run_reference  # noqa: E402

SEED, B, S, G, HP, WP = 11, 2, 96, 8, 32, 32


def main(path: str) -> None:
    bt = make_batch(SEED, B, S)
    ref = run_reference(bt, G, HP, WP)
    np.savez_compressed(path, img=ref["c0.img"].astype(np.float16), n_gt=ref["c0.n_gt"],
                        box=ref["c0.box"].reshape(B, G, 4), gt_inst=ref["c0.gt_inst"],
                        mask=ref["c0.mask"].reshape(B, G, -1), ignore=ref["c0.ignore"].reshape(B, -1),
                        case=np.array([SEED, B, S, G, HP, WP], np.int32))
    print("wrote", path)


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "augment_golden.npz"))
