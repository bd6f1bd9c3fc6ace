"""Llama-2-architecture decoder stack with every linear on the W4A4 path: the prefill workload of the
benchmark (random-init weights, batch 1 x seqlen token ids).

The reference applies its QuantLinear to the linears of a Hugging Face LlamaForCausalLM
(core/model_ops.py:3-6 walks model.model.layers; core/linear.py:48-52 is each wrapped linear). This
module builds the same architecture directly around this package's QuantLinear so that a prefill can
run without the transformers model code or a checkpoint:

    h = embed[ids]
    per layer:  x = RMSNorm(h)
                q, k, v = Wq x, Wk x, Wv x       one rotate+quantize of x shared by the three GEMMs
                q, k = RoPE(q), RoPE(k)
                a = causal attention(q, k, v)      bf16 (torch scaled_dot_product_attention)
                h = h + Wo a                       residual added in the GEMM epilogue
                x = RMSNorm(h)
                g, u = Wg x, Wu x                  one rotate+quantize shared by the two GEMMs
                h = h + Wd (silu(g) * u)           residual added in the GEMM epilogue
    logits = Wlm RMSNorm(h)

All seven projections of every layer and the LM head are W4A4 (symmetric per-token activations,
online Hadamard rotation, symmetric per-channel int4 weights). RMSNorm, RoPE and the SiLU gate are
single-pass bf16 kernels of this package (ops.rmsnorm / rope_ / silu_mul, the same rounding steps as
the torch expressions rms_norm / apply_rope below, which the tests compare them with); causal
attention is torch's scaled_dot_product_attention in bf16.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import ops
from .linear import QuantConfig, QuantLinear


@dataclass
class LlamaConfig:
    vocab: int = 32000
    hidden: int = 4096
    heads: int = 32
    kv_heads: int = 32
    intermediate: int = 11008
    layers: int = 32
    rope_theta: float = 10000.0
    eps: float = 1e-5

    @property
    def head_dim(self) -> int:
        return self.hidden // self.heads


def random_quant_linear(N: int, K: int, gen: torch.Generator, device, std: float = 0.02) -> QuantLinear:
    """A prepared W4A4 QuantLinear with N(0, std) bf16 weights (only the packed weight is kept)."""
    base = torch.nn.Linear(K, N, bias=False, dtype=torch.bfloat16, device=device)
    with torch.no_grad():
        base.weight.copy_((torch.randn(N, K, generator=gen, device=device) * std).to(torch.bfloat16))
    ql = QuantLinear(base, QuantConfig())
    ql.enabled = True
    ql.prepare()
    base.weight.data = torch.empty(0, dtype=torch.bfloat16, device=device)
    return ql


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)).to(x.dtype) * weight


def rope_tables(seq: int, head_dim: int, theta: float, device) -> tuple[torch.Tensor, torch.Tensor]:
    inv = 1.0 / (theta ** (torch.arange(0, head_dim, 2, device=device, dtype=torch.float32) / head_dim))
    f = torch.outer(torch.arange(seq, device=device, dtype=torch.float32), inv)
    emb = torch.cat((f, f), dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def apply_rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [S, H, D]; rotate-half form of rotary embeddings."""
    d = x.shape[-1] // 2
    rot = torch.cat((-x[..., d:], x[..., :d]), dim=-1)
    return x * cos[:, None, :] + rot * sin[:, None, :]


class DecoderLayer:
    def __init__(self, cfg: LlamaConfig, gen: torch.Generator, device):
        H, I, kv = cfg.hidden, cfg.intermediate, cfg.kv_heads * cfg.head_dim
        self.cfg = cfg
        self.q = random_quant_linear(H, H, gen, device)
        self.k = random_quant_linear(kv, H, gen, device)
        self.v = random_quant_linear(kv, H, gen, device)
        self.o = random_quant_linear(H, H, gen, device)
        self.gate = random_quant_linear(I, H, gen, device)
        self.up = random_quant_linear(I, H, gen, device)
        self.down = random_quant_linear(H, I, gen, device)
        self.norm1 = (1.0 + 0.1 * torch.randn(H, generator=gen, device=device)).to(torch.bfloat16)
        self.norm2 = (1.0 + 0.1 * torch.randn(H, generator=gen, device=device)).to(torch.bfloat16)

    def __call__(self, h: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        cfg = self.cfg
        S = h.shape[0]
        x = ops.rmsnorm(h, self.norm1, cfg.eps)
        qx = self.q.quantize_input(x)
        q = self.q.forward_quantized(qx, S).view(S, cfg.heads, cfg.head_dim)
        k = self.k.forward_quantized(qx, S).view(S, cfg.kv_heads, cfg.head_dim)
        v = self.v.forward_quantized(qx, S).view(S, cfg.kv_heads, cfg.head_dim)
        ops.rope_(q, k, cos, sin)
        a = F.scaled_dot_product_attention(q.transpose(0, 1)[None], k.transpose(0, 1)[None], v.transpose(0, 1)[None],
                                           is_causal=True, enable_gqa=cfg.kv_heads != cfg.heads)
        a = a[0].transpose(0, 1).reshape(S, cfg.hidden)
        h = self.o.forward_quantized(self.o.quantize_input(a), S, residual=h)
        x = ops.rmsnorm(h, self.norm2, cfg.eps)
        gx = self.gate.quantize_input(x)
        g = self.gate.forward_quantized(gx, S)
        u = self.up.forward_quantized(gx, S)
        m = ops.silu_mul(g, u)
        return self.down.forward_quantized(self.down.quantize_input(m), S, residual=h)


class LlamaW4A4:
    """Random-init Llama-2 stack (LlamaConfig) on one GPU; __call__(ids [S]) -> logits [S, vocab] bf16."""

    def __init__(self, cfg: LlamaConfig, device, seed: int = 0):
        self.cfg = cfg
        self.device = torch.device(device)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(seed)
        self.embed = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=self.device) * 0.02).to(torch.bfloat16)
        self.layers = [DecoderLayer(cfg, gen, self.device) for _ in range(cfg.layers)]
        self.norm = (1.0 + 0.1 * torch.randn(cfg.hidden, generator=gen, device=self.device)).to(torch.bfloat16)
        self.lm_head = random_quant_linear(cfg.vocab, cfg.hidden, gen, self.device)
        self._rope = {}

    def rope(self, S: int):
        if S not in self._rope:
            self._rope[S] = rope_tables(S, self.cfg.head_dim, self.cfg.rope_theta, self.device)
        return self._rope[S]

    @torch.no_grad()
    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        S = ids.shape[0]
        cos, sin = self.rope(S)
        h = self.embed[ids]
        for layer in self.layers:
            h = layer(h, cos, sin)
        x = ops.rmsnorm(h, self.norm, self.cfg.eps)
        return self.lm_head.forward_quantized(self.lm_head.quantize_input(x), S)

    def graph(self, S: int) -> "PrefillGraph":
        """The prefill of S tokens captured once as a CUDA graph (see PrefillGraph)."""
        return PrefillGraph(self, S)

    def linear_ops(self, S: int) -> float:
        """Integer ops of all W4A4 GEMMs of one prefill of S tokens (2 * S * N * K each)."""
        c = self.cfg
        kv = c.kv_heads * c.head_dim
        per_layer = 2 * S * (c.hidden * c.hidden * 2 + 2 * kv * c.hidden + 3 * c.intermediate * c.hidden)
        return float(per_layer * c.layers + 2 * S * c.vocab * c.hidden)


class PrefillGraph:
    """One CUDA graph holding a whole prefill of S tokens: every kernel of __call__ (rotate+quantize,
    W4A4 GEMMs, RMSNorm, RoPE, attention, SiLU gate, LM head) recorded once and replayed without the
    host issuing each op. The ids are copied into a static buffer, and the logits come back in a
    static buffer that the next replay overwrites. One eager pass runs first on a side stream: the
    first call per device and K builds the rotate+quantize operand, which cannot be captured."""

    def __init__(self, model: LlamaW4A4, S: int):
        dev = model.device
        self.ids = torch.zeros(S, dtype=torch.long, device=dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        with torch.cuda.stream(side):
            model(self.ids)
        torch.cuda.current_stream(dev).wait_stream(side)
        torch.cuda.synchronize(dev)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph):
            self.logits = model(self.ids)

    def __call__(self, ids: torch.Tensor) -> torch.Tensor:
        self.ids.copy_(ids)
        self.graph.replay()
        return self.logits
