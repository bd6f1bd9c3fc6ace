"""Generates tests/golden/golden_v1.npz, golden_transforms_v1.npz and golden_extra_v1.npz from the REFERENCE's
own Python code.

Run in a container where the reference checkout is available (its path is the
first argument, default ../../reference relative to the repository root's
parent). It imports core.quantization and core.linear from that checkout and
records their outputs on seeded inputs produced by dscquant_b200.synthetic, so
the fixtures pin both the CPU oracle (oracle/oracle.py) and the CUDA kernels to
the reference without needing the reference at test time.

    python tests/golden/make_golden.py /path/to/reference [main] [transforms] [extras]
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

from dscquant_b200 import synthetic  # noqa: E402


def main(ref: str) -> None:
    import torch
    from torch import nn

    sys.path.insert(0, ref)
    from core import quantization as Q  # reference
    from core.linear import QuantLinear  # reference

    torch.manual_seed(0)
    out = {"torch_version": np.array(torch.__version__)}

    def bf16(bits):
        return torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16)

    def bits(t):
        return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)

    # -- quantizer functions on a ragged shape (odd K) --------------------------------
    xq = synthetic.activations_bf16(13, 201, seed=11)
    wq = synthetic.weights_bf16(96, 201, seed=12)
    # crafted rows: exact .5 ties after division by the scale (amax = 7 -> scale = 1)
    tie = np.zeros((2, 201), np.float32)
    tie[0, :8] = [7.0, 0.5, 1.5, 2.5, -0.5, -2.5, 3.5, -6.5]
    tie[1, :8] = [-7.0, 4.5, 5.5, 6.5, -1.5, -3.5, -4.5, 0.25]
    wq = np.concatenate([wq, synthetic._to_bf16_bits(tie)], axis=0)
    xq = np.concatenate([xq, synthetic._to_bf16_bits(tie)], axis=0)
    out["q_x"] = xq
    out["q_w"] = wq
    for clip in (1.0, 0.75):
        tag = str(clip).replace(".", "p")
        code, scale = Q.weight_codes(bf16(wq), 4, clip)
        out[f"wc_code_{tag}"] = code.to(torch.int8).numpy()
        out[f"wc_scale_{tag}"] = scale.numpy()
        code, scale, zero = Q.activation_codes(bf16(xq), 4, clip)
        out[f"ac_code_{tag}"] = code.to(torch.int8).numpy()
        out[f"ac_scale_{tag}"] = scale.numpy()
        out[f"ac_zero_{tag}"] = zero.numpy()
        out[f"qw_{tag}"] = bits(Q.quantize_weight(bf16(wq), 4, clip))
        out[f"qa_{tag}"] = bits(Q.quantize_activation(bf16(xq), 4, clip))
    codes_w = Q.weight_codes(bf16(wq), 4, 1.0)[0]
    packed = Q.pack_int4(codes_w)
    out["pack_codes"] = codes_w.to(torch.int8).numpy()
    out["pack_bytes"] = packed.numpy()
    out["unpack_codes"] = Q.unpack_int4(packed, 201).numpy()

    # -- QuantLinear.forward (reference fake-quant path, as shipped) -------------------
    cfg = types.SimpleNamespace(activation_bits=4, weight_bits=4)
    for name, (M, K, N, bias) in {"lin_a": (16, 256, 128, True), "lin_b": (7, 320, 96, False),
                                  "lin_cfg0": (16, 4096, 4096, False)}.items():
        x = synthetic.activations_bf16(M, K, seed=100 + M)
        w = synthetic.weights_bf16(N, K, seed=200 + N)
        base = nn.Linear(K, N, bias=bias, dtype=torch.bfloat16)
        with torch.no_grad():
            base.weight.copy_(bf16(w))
            if bias:
                b = synthetic.weights_bf16(1, N, seed=300 + N, std=0.5)[0]
                base.bias.copy_(bf16(b))
                out[f"{name}_bias"] = b
        ql = QuantLinear(base, cfg)
        ql.enabled = True
        with torch.no_grad():
            y = ql(bf16(x))
        out[f"{name}_shape"] = np.array([M, K, N, int(bias)])
        out[f"{name}_y"] = bits(y)
        if K <= 512:
            out[f"{name}_x"] = x
            out[f"{name}_w"] = w

    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_v1.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


def transforms(ref: str) -> None:
    """golden_transforms_v1.npz: the reference's Rotation / Scaling transforms (core/transforms.py) and
    QuantLinear.transformed() (core/linear.py:22-46) on seeded parameters: per-head rotation matrices, the
    absorbed v / o weights (with a GQA repeat) and the scaled up / down weights."""
    import torch
    from torch import nn

    sys.path.insert(0, ref)
    from core.linear import QuantLinear  # reference
    from core.transforms import Rotation, Scaling  # reference

    g = torch.Generator().manual_seed(1234)
    out = {"torch_version": np.array(torch.__version__)}

    def bits(t):
        return t.detach().contiguous().view(torch.int16).numpy().view(np.uint16)

    def lin(n, k, bias, seed):
        base = nn.Linear(k, n, bias=bias, dtype=torch.bfloat16)
        with torch.no_grad():
            base.weight.copy_(torch.from_numpy(synthetic.weights_bf16(n, k, seed=seed).view(np.int16)).view(torch.bfloat16))
            if bias:
                base.bias.copy_(torch.randn(n, generator=g).to(torch.bfloat16))
        return base

    cfg = types.SimpleNamespace(activation_bits=4, weight_bits=4)
    heads, hd, repeat = 2, 128, 2
    rot = Rotation(heads, hd)
    rot.set_basis("rec", torch.linalg.qr(torch.randn(rot.dimension, 3, generator=g))[0])
    rot.set_basis("sid", torch.randn(rot.dimension, 2, generator=g) * 0.02)
    with torch.no_grad():
        rot.alpha.copy_(torch.randn(3, generator=g))
        rot.beta.copy_(torch.randn(2, generator=g))
        R = rot.matrices()
    out["rot_matrices"] = R.numpy()
    v = lin(heads * hd, 64, True, 400)
    o = lin(48, heads * repeat * hd, False, 401)
    qv = QuantLinear(v, cfg, interface=rot, role="v")
    qo = QuantLinear(o, cfg, interface=rot, role="o", repeat=repeat)
    with torch.no_grad():
        wv, bv = qv.transformed()
        wo, _ = qo.transformed()
    out.update(v_w=bits(v.weight), v_b=bits(v.bias), v_w_t=bits(wv), v_b_t=bits(bv), o_w=bits(o.weight),
               o_w_t=bits(wo), o_repeat=np.array(repeat))
    sc = Scaling(96)
    sc.set_basis("rec", torch.randn(96, 2, generator=g) * 0.3)
    with torch.no_grad():
        sc.alpha.copy_(torch.randn(2, generator=g))
        s_diag = sc.diagonal()
    out["scale_diag"] = s_diag.numpy()
    up = lin(96, 40, True, 402)
    down = lin(30, 96, False, 403)
    with torch.no_grad():
        wu, bu = QuantLinear(up, cfg, interface=sc, role="up").transformed()
        wd, _ = QuantLinear(down, cfg, interface=sc, role="down").transformed()
    out.update(up_w=bits(up.weight), up_b=bits(up.bias), up_w_t=bits(wu), up_b_t=bits(bu), down_w=bits(down.weight),
               down_w_t=bits(wd))
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_transforms_v1.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


def extras(ref: str) -> None:
    """golden_extra_v1.npz: ste_round (core/quantization.py:4-5) forward values and gradients on crafted
    ties, signed zeros and large values; and Rotation.matrices() / Scaling.diagonal()
    (core/transforms.py:42-52, 71-72) together with the buffers and parameters that define them
    (rec_basis, sid_basis, alpha, beta), so a restatement can be pinned from the state alone."""
    import torch

    sys.path.insert(0, ref)
    from core.quantization import ste_round  # reference
    from core.transforms import Rotation, Scaling  # reference

    out = {"torch_version": np.array(torch.__version__)}
    g = torch.Generator().manual_seed(4321)
    crafted = torch.tensor([0.5, 1.5, 2.5, -0.5, -1.5, -2.5, -0.4, -0.0, 0.0, 0.49999997, 7.5, -7.5, 3.0e6 + 0.5,
                            -8.5, 1e-30, -1e-30, 12582912.5, 16777215.0, 2.0 ** 23 + 1.0], dtype=torch.float32)
    x = torch.cat([crafted, torch.randn(1000, generator=g) * 10, torch.rand(64, generator=g).floor() + 0.5])
    xr = x.clone().requires_grad_(True)
    y = ste_round(xr)
    w = torch.randn(x.shape, generator=g)
    (y * w).sum().backward()
    out.update(ste_x=x.numpy(), ste_y=y.detach().numpy(), ste_w=w.numpy(), ste_grad=xr.grad.numpy())

    heads, hd = 3, 16
    rot = Rotation(heads, hd)
    rot.set_basis("rec", torch.linalg.qr(torch.randn(rot.dimension, 4, generator=g))[0])
    rot.set_basis("sid", torch.randn(rot.dimension, 3, generator=g) * 0.05)
    with torch.no_grad():
        rot.alpha.copy_(torch.randn(4, generator=g) * 2)
        rot.beta.copy_(torch.randn(3, generator=g))
        R = rot.matrices()
    out.update(rot_heads=np.array(heads), rot_head_dim=np.array(hd), rot_rec_basis=rot.rec_basis.numpy(),
               rot_sid_basis=rot.sid_basis.numpy(), rot_alpha=rot.alpha.detach().numpy(),
               rot_beta=rot.beta.detach().numpy(), rot_R=R.numpy())
    sc = Scaling(80)
    sc.set_basis("rec", torch.randn(80, 3, generator=g) * 0.3)
    sc.set_basis("sid", torch.randn(80, 2, generator=g) * 0.1)
    with torch.no_grad():
        sc.alpha.copy_(torch.randn(3, generator=g))
        sc.beta.copy_(torch.randn(2, generator=g))
        s_diag = sc.diagonal()
    out.update(sc_rec_basis=sc.rec_basis.numpy(), sc_sid_basis=sc.sid_basis.numpy(), sc_alpha=sc.alpha.detach().numpy(),
               sc_beta=sc.beta.detach().numpy(), sc_diag=s_diag.numpy())
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden_extra_v1.npz")
    np.savez_compressed(path, **out)
    print("wrote", path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    ref_dir = sys.argv[1] if len(sys.argv) > 1 else os.path.join(os.path.dirname(ROOT), "reference")
    which = sys.argv[2:] or ["main", "transforms", "extras"]
    if "main" in which:
        main(ref_dir)
    if "transforms" in which:
        transforms(ref_dir)
    if "extras" in which:
        extras(ref_dir)
