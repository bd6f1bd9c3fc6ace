"""QuantLinear drop-in on the GPU.

* Reference semantics (reference-style config: asymmetric per-token codes, no rotation) against the
  reference's own QuantLinear.forward outputs (tests/golden): relative Frobenius error <= 1e-2.
* Benchmark scheme (QuantConfig(): symmetric codes + online Hadamard rotation) against the oracle's
  float64 fake-quant restatement: relative Frobenius error <= 1e-2; max-abs error reported."""
import types

import numpy as np
import pytest
import torch
from torch import nn

from dscquant_b200 import synthetic

pytestmark = pytest.mark.gpu
TOL = 1e-2


def _f32(bits):
    return (np.asarray(bits, np.uint16).astype(np.uint32) << 16).view(np.float32)


def _tbf(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


def _linear(w_bits, b_bits, dev):
    N, K = w_bits.shape
    base = nn.Linear(K, N, bias=b_bits is not None, dtype=torch.bfloat16, device=dev)
    with torch.no_grad():
        base.weight.copy_(_tbf(w_bits, dev))
        if b_bits is not None:
            base.bias.copy_(_tbf(b_bits, dev))
    return base


@pytest.mark.parametrize("name", ["lin_a", "lin_b", "lin_cfg0"])
def test_reference_semantics_match_reference_output(golden, cuda_device, name):
    from dscquant_b200 import QuantLinear

    M, K, N, has_bias = (int(v) for v in golden[f"{name}_shape"])
    x = golden.get(f"{name}_x", None)
    w = golden.get(f"{name}_w", None)
    if x is None:
        x = synthetic.activations_bf16(M, K, seed=100 + M)
        w = synthetic.weights_bf16(N, K, seed=200 + N)
    b = golden[f"{name}_bias"] if has_bias else None
    ql = QuantLinear(_linear(w, b, cuda_device), types.SimpleNamespace(activation_bits=4, weight_bits=4))
    ql.enabled = True
    y = ql(_tbf(x, cuda_device)).float().cpu().numpy()
    ref = _f32(golden[f"{name}_y"])
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    print(f"{name}: rel_fro={rel:.3e} max_abs={np.abs(y - ref).max():.3e}")
    assert rel <= TOL


def _oracle_fake_quant(oracle, x_bits, w_bits, b_bits=None):
    y = oracle.rotate(_f32(x_bits))
    wr = oracle.rotate(_f32(w_bits))
    cx, sx = oracle.activation_codes_sym(y)
    cw, sw = oracle.weight_codes(wr)
    out = (cx.astype(np.float64) * sx) @ (cw.astype(np.float64) * sw).T
    if b_bits is not None:
        out = out + _f32(b_bits)[None, :]
    return out


@pytest.mark.parametrize("M,K,N", [(16, 4096, 4096), (128, 11008, 512), (64, 14336, 256), (5, 4096, 11008)])
def test_symmetric_rotated_matches_oracle(oracle, cuda_device, M, K, N):
    from dscquant_b200 import QuantConfig, QuantLinear

    x = synthetic.activations_bf16(M, K, seed=M)
    w = synthetic.weights_bf16(N, K, seed=N)
    ql = QuantLinear(_linear(w, None, cuda_device), QuantConfig())
    ql.enabled = True
    y = ql(_tbf(x, cuda_device)).float().cpu().numpy()
    ref = _oracle_fake_quant(oracle, x, w)
    rel = np.linalg.norm(y - ref) / np.linalg.norm(ref)
    dense = _f32(x).astype(np.float64) @ _f32(w).astype(np.float64).T
    rel_dense = np.linalg.norm(y - dense) / np.linalg.norm(dense)
    print(f"M={M} K={K} N={N}: rel_fro vs fake-quant={rel:.3e} max_abs={np.abs(y - ref).max():.3e} "
          f"(vs unquantized: {rel_dense:.3e})")
    assert rel <= TOL


def test_rotated_integer_path_exact(oracle, cuda_device):
    """GPU accumulators of the module equal the oracle's integer GEMM on the module's own packed operands."""
    from dscquant_b200 import QuantConfig, QuantLinear, ops

    M, K, N = 32, 11008, 384
    x = synthetic.activations_bf16(M, K, seed=1)
    w = synthetic.weights_bf16(N, K, seed=2)
    ql = QuantLinear(_linear(w, None, cuda_device), QuantConfig())
    ql.enabled = True
    ql.prepare()
    q = ops.rowquant(_tbf(x, cuda_device), "act_sym", rotate=True, KP=ql._prep["KP"])
    out, raw = ops.w4a4_gemm(q.packed, ql._prep["packed"], q.scales, ql._prep["sw"], return_raw=True)
    a = q.packed.cpu().numpy()
    b = ql._prep["packed"].cpu().numpy()
    ref_raw = oracle.gemm_s4(a, b, M, N, ql._prep["KP"])
    np.testing.assert_array_equal(raw.cpu().numpy(), ref_raw)
    ref = oracle.epilogue(ref_raw, q.scales.cpu().numpy(), ql._prep["sw"].cpu().numpy())
    np.testing.assert_array_equal(out.cpu().view(torch.int16).numpy().view(np.uint16), oracle.f32_to_bf16_bits(ref))
    y = ql(_tbf(x, cuda_device))
    assert torch.equal(y, out)


def test_leading_dims_bias_and_prepare_once(cuda_device):
    from dscquant_b200 import QuantConfig, QuantLinear

    K, N = 4096, 256
    w = synthetic.weights_bf16(N, K, seed=5)
    b = synthetic.weights_bf16(1, N, seed=6, std=0.5)[0]
    ql = QuantLinear(_linear(w, b, cuda_device), QuantConfig())
    ql.enabled = True
    x = torch.randn(2, 5, K, device=cuda_device, dtype=torch.bfloat16)
    y3 = ql(x)
    packed = ql._prep["packed"]
    y2 = ql(x.reshape(10, K))
    assert y3.shape == (2, 5, N) and ql._prep["packed"] is packed
    assert torch.equal(y3.reshape(10, N), y2)
    ql.enabled = False
    torch.testing.assert_close(ql(x), ql.base(x))


def test_fp16_and_fp32_inputs(cuda_device):
    from dscquant_b200 import QuantConfig, QuantLinear

    for dt in (torch.float16, torch.float32):
        base = nn.Linear(256, 64, dtype=dt, device=cuda_device)
        ql = QuantLinear(base, QuantConfig())
        ql.enabled = True
        x = torch.randn(3, 256, dtype=dt, device=cuda_device)
        y = ql(x)
        assert y.dtype == dt
        rel = (y.float() - base(x).float()).norm() / base(x).float().norm()
        assert rel < 0.25


def test_prepared_state_roundtrip_gpu(cuda_device):
    """A layer loaded from another layer's prepared state produces bit-identical outputs."""
    from dscquant_b200 import QuantConfig, QuantLinear

    K, N = 4096, 384
    w = synthetic.weights_bf16(N, K, seed=9)
    a = QuantLinear(_linear(w, None, cuda_device), QuantConfig())
    a.enabled = True
    st = a.prepared_state()
    b = QuantLinear(nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=cuda_device), QuantConfig())
    b.enabled = True
    b.load_prepared(st)
    x = torch.randn(33, K, device=cuda_device, dtype=torch.bfloat16)
    assert torch.equal(a(x), b(x))


def test_host_pipeline_matches_forward(cuda_device):
    """HostPipeline (pinned host in/out, copies overlapped with the kernels on three streams) returns the
    same bits as QuantLinear.forward on device tensors, over repeated calls that reuse its buffers."""
    from dscquant_b200 import QuantConfig, QuantLinear
    from dscquant_b200.hostio import HostPipeline

    shapes = [(4096, 512), (4096, 1024), (11008, 256)]
    mods, h_in, h_out, refs = [], [], [], []
    for i, (K, N) in enumerate(shapes):
        ql = QuantLinear(_linear(synthetic.weights_bf16(N, K, seed=40 + i), None, cuda_device), QuantConfig())
        ql.enabled = True
        x = torch.randn(96, K, device=cuda_device, dtype=torch.bfloat16)
        refs.append(ql(x).cpu())
        mods.append(ql)
        h_in.append(x.cpu().pin_memory())
        h_out.append(torch.empty((96, N), dtype=torch.bfloat16).pin_memory())
    pipe = HostPipeline(cuda_device)
    for _ in range(3):
        for h in h_out:
            h.zero_()
        pipe.run(mods, h_in, h_out)
        pipe.synchronize()
        for h, r in zip(h_out, refs):
            assert torch.equal(h, r)
    with pytest.raises(ValueError):
        pipe.run(mods, [t.clone() for t in h_in], h_out)  # not pinned


def test_host_pipeline_shared_input(cuda_device):
    """A host input shared by several modules (q/k/v style) is copied once and still gives every
    module's forward bits, over repeated calls that reuse the device buffers."""
    from dscquant_b200 import QuantConfig, QuantLinear
    from dscquant_b200.hostio import HostPipeline

    K = 4096
    x = torch.randn(80, K, device=cuda_device, dtype=torch.bfloat16)
    x2 = torch.randn(80, K, device=cuda_device, dtype=torch.bfloat16)
    h_x, h_x2 = x.cpu().pin_memory(), x2.cpu().pin_memory()
    mods, h_in, h_out, refs = [], [], [], []
    for i, (N, src, hsrc) in enumerate([(512, x, h_x), (256, x, h_x), (768, x2, h_x2), (256, x, h_x)]):
        ql = QuantLinear(_linear(synthetic.weights_bf16(N, K, seed=60 + i), None, cuda_device), QuantConfig())
        ql.enabled = True
        refs.append(ql(src).cpu())
        mods.append(ql)
        h_in.append(hsrc)
        h_out.append(torch.empty((80, N), dtype=torch.bfloat16).pin_memory())
    pipe = HostPipeline(cuda_device)
    for _ in range(3):
        for h in h_out:
            h.zero_()
        pipe.run(mods, h_in, h_out)
        pipe.synchronize()
        for h, r in zip(h_out, refs):
            assert torch.equal(h, r)


def test_int8_activation_path_same_bits(cuda_device):
    """QuantLinear with int8_activations (A8 GEMM above 64 tokens) returns the packed path's bits."""
    from dscquant_b200 import QuantConfig, QuantLinear

    K, N = 4096, 512
    w = synthetic.weights_bf16(N, K, seed=12)
    ql = QuantLinear(_linear(w, None, cuda_device), QuantConfig())
    ql.enabled = True
    x = torch.randn(300, K, device=cuda_device, dtype=torch.bfloat16)
    y_packed = ql(x)
    ql.int8_activations = True
    y_a8 = ql(x)
    assert torch.equal(y_packed, y_a8)


class _HeadRotation:
    """Stand-in for core/transforms.py Rotation: the attributes QuantLinear reads (heads, head_dim, matrices())."""

    def __init__(self, R):
        self.heads, self.head_dim, self._R = R.shape[0], R.shape[1], R

    def matrices(self):
        return self._R


def test_online_head_rotation_matches_absorbed(cuda_device):
    """Role 'o' with online_head_rotation: input rotated per head inside the quantize kernel, weight W_o R as in
    core/linear.py:34-37. The module output equals the kernel's codes fed to the GEMM (bit-exact wiring); against
    the float product it is as accurate as the absorbed path fed with the already-rotated input (what W_v R^T
    would produce; that path quantises bf16(x R), the online one the f32 product, so the two differ by int4
    rounding-boundary flips, not by a common reference). Role 'v' keeps its plain weight."""
    from dscquant_b200 import QuantConfig, QuantLinear, ops

    heads, M, N = 8, 96, 512
    K = 128 * heads
    g = torch.Generator().manual_seed(11)
    a = torch.randn(heads, 128, 128, generator=g, dtype=torch.float64) * 0.05
    R = torch.matrix_exp(a - a.transpose(1, 2)).float().to(cuda_device)
    rot = _HeadRotation(R)
    base = _linear(synthetic.weights_bf16(N, K, seed=70), None, cuda_device)
    on = QuantLinear(base, QuantConfig(online_rotation=False, online_head_rotation=True), interface=rot, role="o")
    off = QuantLinear(base, QuantConfig(online_rotation=False), interface=rot, role="o")
    on.enabled = off.enabled = True
    x = _tbf(synthetic.activations_bf16(M, K, seed=71), cuda_device)
    x_rot = torch.einsum("thd,hde->the", x.float().reshape(M, heads, 128), R).reshape(M, K).to(torch.bfloat16)
    y_on, y_off = on(x), off(x_rot)
    q = ops.rowquant_headrot(x, *on._prep["head_rot"], "act_sym")
    assert torch.equal(y_on, ops.w4a4_gemm(q.packed, on._prep["packed"], q.scales, on._prep["sw"]))
    y_fp = x.float() @ base.weight.float().T
    rel = lambda a, b: (torch.linalg.norm(a.float() - b) / torch.linalg.norm(b)).item()  # noqa: E731
    e_on, e_off = rel(y_on, y_fp), rel(y_off, y_fp)
    print(f"online head rotation: rel_fro vs float {e_on:.3e} (absorbed path {e_off:.3e})")
    # the synthetic activations carry x20 outlier channels that a within-head rotation barely spreads, so plain
    # W4A4 error is large here; the check is that the online path is as accurate as the absorbed one
    assert e_on < 1.0 and e_on <= 1.05 * e_off + 1e-3
    v = QuantLinear(base, QuantConfig(online_rotation=False, online_head_rotation=True), interface=rot, role="v")
    assert torch.equal(v.transformed()[0], base.weight)
    state = on.prepared_state()
    re = QuantLinear(base, QuantConfig(online_rotation=False, online_head_rotation=True), interface=rot, role="o")
    re.enabled = True
    re.load_prepared(state)
    assert torch.equal(re(x), on(x))


class _Scaling:
    """Stand-in for core/transforms.py Scaling: diagonal() only."""

    def __init__(self, s):
        self._s = s

    def diagonal(self):
        return self._s


def test_online_scaling_in_epilogue(cuda_device):
    """Role 'up' with online_scaling: codes of the plain weight, channel scales sw / s applied by the GEMM epilogue
    (bit-exact wiring), output as accurate as the reference's absorbed W / s path."""
    from dscquant_b200 import QuantConfig, QuantLinear, ops

    M, K, N = 64, 1024, 384
    g = torch.Generator().manual_seed(3)
    s = torch.exp(torch.randn(N, generator=g) * 0.3).to(cuda_device)
    base = _linear(synthetic.weights_bf16(N, K, seed=80), synthetic.weights_bf16(1, N, seed=81, std=0.5)[0],
                   cuda_device)
    scaling = _Scaling(s)  # QuantLinear holds its interface by weakref (core/linear.py:15): keep it alive
    on = QuantLinear(base, QuantConfig(online_rotation=False, online_scaling=True), interface=scaling, role="up")
    off = QuantLinear(base, QuantConfig(online_rotation=False), interface=scaling, role="up")
    assert on.online_up_scaling and not off.online_up_scaling
    plain = QuantLinear(base, QuantConfig(online_rotation=False))
    for m in (on, off, plain):
        m.enabled = True
        m.prepare()
    assert torch.equal(on._prep["packed"], plain._prep["packed"])
    assert torch.equal(on._prep["sw"], plain._prep["sw"] / s)
    x = _tbf(synthetic.activations_bf16(M, K, seed=82), cuda_device)
    y_on, y_off = on(x), off(x)
    q = ops.rowquant(x, "act_sym", KP=K)
    bias = (base.bias.float() / s).to(torch.bfloat16)
    assert torch.equal(y_on, ops.w4a4_gemm(q.packed, on._prep["packed"], q.scales, on._prep["sw"], bias=bias))
    y_ref = (x.float() @ base.weight.float().T) / s + bias.float()
    rel = lambda a, b: (torch.linalg.norm(a.float() - b) / torch.linalg.norm(b)).item()  # noqa: E731
    e_on, e_off = rel(y_on, y_ref), rel(y_off, y_ref)
    print(f"online scaling: rel_fro vs float {e_on:.3e} (absorbed path {e_off:.3e})")
    assert e_on <= 1.05 * e_off + 1e-3
