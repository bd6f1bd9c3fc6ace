"""Generates tests/golden/golden_refkernel_v1.npz by running the REFERENCE's own CUDA quantizer on a GPU.

The reference's kernel/w4a4.cu, compiled unmodified by oracle/build_ref.py into oracle/_ref/, runs its
``quantize`` (quantize_cuda, kernel/w4a4.cu:164-187) on seeded fp16 / fp32 inputs and several clip
values, fused and unfused; the inputs and the packed bytes, scales and zero points it returns are
saved. The fixture pins the oracle's restatement of the reference kernel's arithmetic (asymmetric
mode ACT_ASYM, tests/test_oracle.py) on machines without a GPU. It was produced on a B200 with
the nvcc 12.9 build of the reference (nvcc's default floating-point contraction):

    python tests/golden/make_golden_refkernel.py [output.npz]
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

CASES = [  # (M, K, dtype, clip)
    (24, 300, "float16", 1.0), (24, 300, "float32", 0.8), (19, 256, "float16", 0.55), (6, 4096, "float32", 0.9),
    (9, 130, "float32", 0.5), (1, 40000, "float16", 0.7), (5, 64, "float32", 1.0),
]


def inputs(M: int, K: int, dtype: str, seed: int):
    import torch

    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g)
    cols = torch.randperm(K, generator=g)[: max(1, K // 100)]
    x[:, cols] *= 20.0
    if M > 2:
        x[1] = x[1].abs()
        x[2] = -x[2].abs()
    if M > 4:  # multiples of a quarter: many y/s + zero sums land exactly on .5
        x[3] = torch.round(x[3] * 4) / 4
        x[4] = torch.round(x[4] * 2) / 2
    return x.to(getattr(torch, dtype))


def main(path: str) -> None:
    import torch

    import build_ref

    ref = build_ref.load()
    dev = torch.device("cuda", 0)
    out = {"torch_version": np.array(torch.__version__), "device": np.array(torch.cuda.get_device_name(dev))}
    for i, (M, K, dtype, clip) in enumerate(CASES):
        x = inputs(M, K, dtype, seed=100 + i).to(dev)
        out[f"c{i}_x"] = x.cpu().numpy()  # in the input dtype (float16 / float32)
        out[f"c{i}_meta"] = np.array([M, K, clip], dtype=np.float64)
        out[f"c{i}_dtype"] = np.array(dtype)
        for fused in (True, False):
            packed, scales, zeros = ref.quantize(x, clip, fused)
            tag = "f" if fused else "u"
            out[f"c{i}_{tag}_packed"] = packed.cpu().numpy()
            out[f"c{i}_{tag}_scales"] = scales.cpu().numpy()
            out[f"c{i}_{tag}_zeros"] = zeros.cpu().numpy()
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.path.join(HERE, "golden_refkernel_v1.npz"))
