"""The Llama-2 prefill harness (dscquant_b200/llama.py) on a small configuration: shared-input projections
(one rotate+quantize feeding q/k/v or gate/up) give the same bits as each QuantLinear's own forward, the
residual added in the GEMM epilogue equals a separate add, and a prefill is finite and deterministic."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_shared_input_projection_matches_forward(cuda_device):
    from dscquant_b200.llama import random_quant_linear

    g = torch.Generator(device=cuda_device).manual_seed(0)
    a = random_quant_linear(384, 1024, g, cuda_device)
    b = random_quant_linear(512, 1024, g, cuda_device)
    x = torch.randn(70, 1024, generator=g, device=cuda_device).to(torch.bfloat16)
    q = a.quantize_input(x)
    assert torch.equal(a.forward_quantized(q, 70), a(x))
    assert torch.equal(b.forward_quantized(q, 70), b(x))
    r = torch.randn(70, 512, generator=g, device=cuda_device).to(torch.bfloat16)
    fused = b.forward_quantized(q, 70, residual=r)
    f32 = b.forward_quantized(q, 70, out_dtype=torch.float32)  # the epilogue value before rounding
    assert torch.equal(fused, (f32 + r.float()).to(torch.bfloat16))  # one rounding of the fp32 sum


def test_small_llama_prefill(cuda_device):
    from dscquant_b200.llama import LlamaConfig, LlamaW4A4

    cfg = LlamaConfig(vocab=512, hidden=1024, heads=8, kv_heads=4, intermediate=2048, layers=2)
    model = LlamaW4A4(cfg, cuda_device, seed=1)
    ids = torch.randint(0, cfg.vocab, (96,), device=cuda_device, generator=torch.Generator(device=cuda_device).manual_seed(2))
    y1 = model(ids)
    y2 = model(ids)
    assert y1.shape == (96, cfg.vocab) and y1.dtype == torch.bfloat16
    assert bool(torch.isfinite(y1.float()).all())
    assert torch.equal(y1, y2)
    assert model.linear_ops(96) > 0


def test_prefill_graph_replay_matches_eager(cuda_device):
    """The CUDA-graph prefill launches the same kernels: its logits equal the eager pass bit for bit, for
    two different token sequences replayed from one graph."""
    from dscquant_b200.llama import LlamaConfig, LlamaW4A4

    cfg = LlamaConfig(vocab=512, hidden=1024, heads=8, kv_heads=4, intermediate=2048, layers=2)
    model = LlamaW4A4(cfg, cuda_device, seed=3)
    gen = torch.Generator(device=cuda_device).manual_seed(4)
    g = model.graph(128)
    for _ in range(2):
        ids = torch.randint(0, cfg.vocab, (128,), device=cuda_device, generator=gen)
        ref = model(ids)
        out = g(ids).clone()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
    del g


def test_prefill_elementwise_ops_match_torch(cuda_device):
    """ops.rmsnorm / rope_ / silu_mul against the torch expressions of the harness: RoPE bit-exact (same
    rounding steps); RMSNorm and the SiLU gate within one bf16 step (the row sum of squares, rsqrt and exp
    may round differently from torch's kernels)."""
    import torch.nn.functional as F

    from dscquant_b200 import ops
    from dscquant_b200.llama import apply_rope, rms_norm, rope_tables

    g = torch.Generator(device=cuda_device).manual_seed(4)
    S, H, D = 300, 12, 128
    x = (torch.randn(S, H * D, generator=g, device=cuda_device) * 3).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(H * D, generator=g, device=cuda_device)).to(torch.bfloat16)
    ref = rms_norm(x, w, 1e-5)
    out = ops.rmsnorm(x, w, 1e-5)
    ulp = (ref.float().abs() * 2 ** -7).clamp_min(1e-30)
    assert bool(((out.float() - ref.float()).abs() <= ulp).all())
    cos, sin = rope_tables(S, D, 10000.0, cuda_device)
    q = torch.randn(S, H, D, generator=g, device=cuda_device).to(torch.bfloat16)
    k = torch.randn(S, 4, D, generator=g, device=cuda_device).to(torch.bfloat16)
    rq, rk = apply_rope(q, cos, sin), apply_rope(k, cos, sin)
    ops.rope_(q, k, cos, sin)
    assert torch.equal(q, rq) and torch.equal(k, rk)
    cos2, sin2 = rope_tables(S, 24, 10000.0, cuda_device)  # D/2 = 12: the one-pair-per-thread kernel
    q2 = torch.randn(S, 3, 24, generator=g, device=cuda_device).to(torch.bfloat16)
    k2 = torch.randn(S, 2, 24, generator=g, device=cuda_device).to(torch.bfloat16)
    rq2, rk2 = apply_rope(q2, cos2, sin2), apply_rope(k2, cos2, sin2)
    ops.rope_(q2, k2, cos2, sin2)
    assert torch.equal(q2, rq2) and torch.equal(k2, rk2)
    a = (torch.randn(S, 1000, generator=g, device=cuda_device) * 4).to(torch.bfloat16)
    b = torch.randn(S, 1000, generator=g, device=cuda_device).to(torch.bfloat16)
    ref = F.silu(a) * b
    out = ops.silu_mul(a, b)
    ulp = (ref.float().abs() * 2 ** -7).clamp_min(1e-30)
    assert bool(((out.float() - ref.float()).abs() <= ulp).all())
