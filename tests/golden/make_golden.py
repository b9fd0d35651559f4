"""Generate golden vectors from the REFERENCE implementation itself.

Runs the reference package's own Triton kernels (``wmma_fwd``, ``wmma_dw``,
``wmma_dx`` and ``transpose_k2s2_fwd/dx/dw`` of rdna4_conv3d) under Triton's
CPU interpreter (``TRITON_INTERPRET=1``) on small seeded inputs and stores
inputs and outputs as ``.npz`` fixtures next to this script. The fixtures pin
the C oracle (tests/test_oracle_golden.py) and the B200 kernels
(tests/test_gpu_parity.py).

Usage (needs the reference checkout, which only exists on the build host):
    python tests/golden/make_golden.py /path/to/reference

Cases follow the reference's own GPU test (tests/test_conv3d.py:47-75 of the
reference: seed 0, fp16 randn x/w/b, randn grad_out), plus pad 0 / pad 2 k3
cases and a k2s2 ConvTranspose3d case, which the reference's tests never pin.
For k3 with pad != 1 the reference's dX is not recorded: its k3 dX reuses the
forward padding (conv3d_wmma.py:1154-1162) and is only correct for pad 1.
"""
from __future__ import annotations

import os
import sys

import numpy as np

OUT_DIR = os.path.dirname(os.path.abspath(__file__))

CONV_CASES = [
    # name,              n, cin, cout, d,  h,  w, k, pad, dx_valid
    ("ref_k3_c5_c7", 2, 5, 7, 9, 11, 13, 3, 1, True),
    ("ref_k1_c24_c1", 2, 24, 1, 8, 16, 16, 1, 0, True),
    ("ref_k3_c24_c24", 1, 24, 24, 8, 16, 16, 3, 1, True),
    ("ref_k3_c1_c24", 1, 1, 24, 8, 16, 16, 3, 1, True),
    ("k3_c16_c8_pad0", 1, 16, 8, 6, 7, 9, 3, 0, False),
    ("k3_c8_c16_pad2", 1, 8, 16, 4, 5, 6, 3, 2, False),
    ("k1_c48_c24", 1, 48, 24, 4, 8, 12, 1, 0, True),
]
TCONV_CASES = [
    # name,             n, cin, cout, d, h, w
    ("tconv_c16_c8", 2, 16, 8, 3, 4, 5),
    ("tconv_c48_c24", 1, 48, 24, 2, 4, 6),
]


def main(ref_root: str) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    os.environ["RDNA4_CONV3D_BACKEND"] = "wmma"
    sys.path.insert(0, os.path.join(ref_root, "src"))
    import torch
    import rdna4_conv3d  # noqa: F401  (the reference package)
    ref = sys.modules["rdna4_conv3d.conv3d_wmma"]

    for name, n, cin, cout, d, h, w, k, pad, dx_valid in CONV_CASES:
        torch.manual_seed(0)
        x = torch.randn(n, cin, d, h, w, dtype=torch.float16)
        wt = torch.randn(cout, cin, k, k, k, dtype=torch.float16)
        b = torch.randn(cout, dtype=torch.float16)
        y = ref.wmma_fwd(x, wt, b, 1, pad)
        go = torch.randn(y.shape, dtype=torch.float16)
        dw = ref.wmma_dw(x, wt, go, 1, pad)
        rec = dict(x=x.numpy(), w=wt.numpy(), b=b.numpy(), go=go.numpy(), y=y.numpy(), dw=dw.numpy(),
                   meta=np.array([n, cin, cout, d, h, w, k, pad], np.int64))
        if dx_valid:
            rec["dx"] = ref.wmma_dx(x, wt, go, 1, pad).numpy()
        np.savez_compressed(os.path.join(OUT_DIR, f"{name}.npz"), **rec)
        print("wrote", name, {kk: v.shape for kk, v in rec.items()})

    for name, n, cin, cout, d, h, w in TCONV_CASES:
        torch.manual_seed(0)
        x = torch.randn(n, cin, d, h, w, dtype=torch.float16)
        wt = torch.randn(cin, cout, 2, 2, 2, dtype=torch.float16)
        b = torch.randn(cout, dtype=torch.float16)
        y = ref.transpose_k2s2_fwd(x, wt, b).contiguous()
        go = torch.randn(y.shape, dtype=torch.float16)
        dx = ref.transpose_k2s2_dx(x.shape, wt, go).contiguous()
        dw = ref.transpose_k2s2_dw(x, wt.shape, go)
        rec = dict(x=x.numpy(), w=wt.numpy(), b=b.numpy(), go=go.numpy(), y=y.numpy(), dx=dx.numpy(),
                   dw=dw.numpy(), meta=np.array([n, cin, cout, d, h, w, 2, 0], np.int64))
        np.savez_compressed(os.path.join(OUT_DIR, f"{name}.npz"), **rec)
        print("wrote", name, {kk: v.shape for kk, v in rec.items()})


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(sys.argv[1])
