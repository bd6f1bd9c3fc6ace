"""Drop-in QuantLinear (core/linear.py:8-52) running the W4A4 CUDA path.

Same constructor, `enabled` flag, clip parameters and `transformed()`
semantics as the reference. Differences, all deliberate:

* the weight is rotated, quantised and packed once (`prepare()`, called
  lazily by the first enabled forward) instead of being re-quantised on every
  call (core/linear.py:52 requantises the full N x K weight per forward);
  call `prepare()` again after changing the weight, the clips or the
  interface;
* the enabled forward runs two kernels: the fused rotate+quantize of the
  activations and the tcgen05 W4A4 GEMM with the dequant epilogue. It accepts
  CUDA tensors only;
* the activation scheme follows the config: a reference-style config (only
  `activation_bits` / `weight_bits`) gives the reference's semantics exactly
  (asymmetric per-token codes, core/quantization.py:13-21, no online rotation);
  `QuantConfig()` gives the symmetric per-token scheme with the online
  Hadamard rotation applied to activations and weights;
* `QuantConfig(online_rotation=False, online_head_rotation=True)` applies the
  per-head Rotation online instead of absorbing it into W_v: role 'v' keeps
  its plain weight, and role 'o' keeps W_o R_h (as core/linear.py:34-37) while
  its input is rotated per head inside the quantize kernel
  (ops.rowquant_headrot). The layer output is the same product in exact
  arithmetic (x R (W_o R)^T = x W_o^T per head);
* `QuantConfig(online_scaling=True)` applies the `Scaling` diagonal of role
  'up' (core/linear.py:40-43: rows of W and the bias divided by s) in the
  GEMM epilogue: the codes come from the plain weight (per-row symmetric codes
  do not change under a per-row scale) and the channel scales become sw / s,
  so the output is the reference's up to the bf16 rounding of W / s that the
  reference applies before quantising. Role 'down' stays absorbed (W diag(s)).
"""
from __future__ import annotations

import weakref
from dataclasses import dataclass

import torch
from torch import nn

from . import ops


@dataclass
class QuantConfig:
    activation_bits: int = 4
    weight_bits: int = 4
    activation_symmetric: bool = True   # scale = absmax/7, codes in [-8, 7]
    online_rotation: bool = True        # y = x (H_a (x) H_b)/sqrt(K) on activations, W' = W (same) offline
    online_head_rotation: bool = False  # per-head Rotation applied to the o-projection's input online
    online_scaling: bool = False        # Scaling of role 'up' applied in the GEMM epilogue (channel scales / s)


class QuantLinear(nn.Module):
    def __init__(self, base: nn.Linear, config, interface=None, role=None, repeat=1):
        super().__init__()
        self.base = base
        self.config = config
        self.role, self.repeat = role, repeat
        self._interface = None if interface is None else weakref.ref(interface)
        self.weight_clip = nn.Parameter(torch.tensor(1.0, device=base.weight.device), requires_grad=False)
        self.activation_clip = nn.Parameter(torch.tensor(1.0, device=base.weight.device), requires_grad=False)
        self.enabled = False
        for param in self.base.parameters():
            param.requires_grad_(False)
        self._prep = None

    # ------------------------------------------------------------------ reference semantics
    def transformed(self):
        """core/linear.py:22-46: absorb the interface (per-head rotation for roles 'v'/'o', diagonal
        scaling otherwise) into (weight, bias)."""
        weight, bias = self.base.weight, self.base.bias
        interface = self._interface() if self._interface else None
        if interface is None:
            return weight, bias
        if hasattr(interface, "matrices"):
            if self.online_heads and self.role == "v":
                return weight, bias  # the o-projection rotates its input online instead
            mats = interface.matrices()
            if self.role == "v":
                shaped = weight.float().reshape(interface.heads, interface.head_dim, -1)
                weight = (mats.transpose(-1, -2) @ shaped).reshape_as(weight).to(weight.dtype)
                if bias is not None:
                    bias = (mats.transpose(-1, -2) @ bias.float().reshape(interface.heads, -1, 1)).flatten().to(
                        bias.dtype)
            elif self.role == "o":
                mats = mats.repeat_interleave(self.repeat, dim=0)
                shaped = weight.float().reshape(weight.shape[0], len(mats), interface.head_dim)
                weight = torch.einsum("ohd,hde->ohe", shaped, mats).reshape_as(weight).to(weight.dtype)
        else:
            scale = interface.diagonal()
            if self.role == "up":
                if not self.online_up_scaling:  # online: the epilogue divides by s (prepare())
                    weight = (weight.float() / scale[:, None]).to(weight.dtype)
                if bias is not None:
                    bias = (bias.float() / scale).to(bias.dtype)
            else:
                weight = (weight.float() * scale[None, :]).to(weight.dtype)
        return weight, bias

    # ------------------------------------------------------------------ W4A4 path
    @property
    def symmetric(self) -> bool:
        return bool(getattr(self.config, "activation_symmetric", False))

    @property
    def rotate(self) -> bool:
        return bool(getattr(self.config, "online_rotation", False))

    @property
    def online_up_scaling(self) -> bool:
        """Scaling of role 'up' applied in the GEMM epilogue (online_scaling)."""
        interface = self._interface() if self._interface else None
        return (bool(getattr(self.config, "online_scaling", False)) and interface is not None and
                hasattr(interface, "diagonal") and not hasattr(interface, "matrices") and self.role == "up")

    @property
    def online_heads(self) -> bool:
        """Per-head Rotation interface applied online (roles 'v' / 'o' with online_head_rotation)."""
        interface = self._interface() if self._interface else None
        return (bool(getattr(self.config, "online_head_rotation", False)) and interface is not None and
                hasattr(interface, "matrices") and self.role in ("v", "o"))

    def _check_bits(self) -> None:
        if int(self.config.activation_bits) != 4 or int(self.config.weight_bits) != 4:
            raise NotImplementedError("the CUDA path implements W4A4 only (activation_bits = weight_bits = 4)")

    @torch.no_grad()
    def prepare(self) -> None:
        """Rotate (optionally), quantise and pack the weight once: packed [N, KP/2] u8, channel scales
        [N] f32 and code sums [N] i32 (for the asymmetric correction, kernel/w4a4.cu:74)."""
        self._check_bits()
        weight, bias = self.transformed()
        if not weight.is_cuda:
            raise RuntimeError("QuantLinear's W4A4 path needs the weight on a CUDA device")
        N, K = weight.shape
        KP = (K + 63) // 64 * 64
        w = weight if weight.dtype in (torch.bfloat16, torch.float16, torch.float32) else weight.float()
        q = ops.rowquant(w.contiguous(), "weight_sym", clip=float(self.weight_clip), rotate=self.rotate, KP=KP,
                         row_sums=True)
        sw = q.scales
        if self.online_up_scaling:  # the diagonal of role 'up' folded into the per-channel epilogue scale
            sw = (sw / self._interface().diagonal().to(device=sw.device, dtype=torch.float32)).contiguous()
        self._prep = dict(packed=q.packed, sw=sw, wsum=q.row_sums, bias=bias, K=K, N=N, KP=KP,
                          aclip=float(self.activation_clip), bias_cache={})
        self._attach_head_rotation()

    def _attach_head_rotation(self) -> None:
        """Role 'o' with online_head_rotation: the (hi, lo) rotation operands of the input quantizer."""
        if not (self.online_heads and self.role == "o"):
            return
        if self.rotate or not self.symmetric:
            raise NotImplementedError("online head rotation needs symmetric activations and online_rotation=False")
        K, KP = self._prep["K"], self._prep["KP"]
        mats = self._interface().matrices().repeat_interleave(self.repeat, dim=0)  # core/linear.py:35
        if mats.shape[1:] != (128, 128) or K != 128 * mats.shape[0] or K != KP:
            raise NotImplementedError("online head rotation needs head_dim 128 and K = heads * 128")
        self._prep["head_rot"] = ops.head_rotation_operands(mats.to(self._prep["packed"].device))

    # int8_activations = True: above A8_MIN_TOKENS tokens the symmetric scheme hands the GEMM int8
    # activation codes (w4a4_gemm_a8) instead of packed nibbles. Same output bits; measured on par with
    # the packed kernel on B200, so it is off by default.
    int8_activations = False
    A8_MIN_TOKENS = 64

    # ------------------------------------------------------------------ packed-weight format
    PREPARED_FORMAT = "dscq-w4a4-v1"

    def prepared_state(self) -> dict:
        """The prepared weight as plain tensors (CPU copies) plus the spec needed to use it:
        packed int4 [N, KP/2] (the reference's packing), channel scales, code sums, bias, and the
        quantisation / rotation settings. `load_prepared` restores it without re-quantising."""
        if self._prep is None:
            self.prepare()
        p = self._prep
        return {
            "format": self.PREPARED_FORMAT,
            "K": p["K"], "N": p["N"], "KP": p["KP"],
            "weight_packed": p["packed"].cpu(), "weight_scales": p["sw"].cpu(), "weight_code_sums": p["wsum"].cpu(),
            "bias": None if p["bias"] is None else p["bias"].detach().cpu(),
            "activation_clip": p["aclip"], "weight_clip": float(self.weight_clip),
            "activation_symmetric": self.symmetric, "online_rotation": self.rotate,
        }

    def load_prepared(self, state: dict) -> None:
        """Installs a `prepared_state()` on this module's device (checks the format and shapes)."""
        if state.get("format") != self.PREPARED_FORMAT:
            raise ValueError(f"unknown prepared-weight format {state.get('format')!r}")
        K, N = self.base.in_features, self.base.out_features
        if (state["K"], state["N"]) != (K, N) or tuple(state["weight_packed"].shape) != (N, state["KP"] // 2):
            raise ValueError("prepared weight does not match this layer's shape")
        if bool(state["activation_symmetric"]) != self.symmetric or bool(state["online_rotation"]) != self.rotate:
            raise ValueError("prepared weight was made for a different activation scheme / rotation setting")
        dev = self.base.weight.device
        bias = state["bias"]
        self._prep = dict(packed=state["weight_packed"].to(dev), sw=state["weight_scales"].to(dev),
                          wsum=state["weight_code_sums"].to(dev), bias=None if bias is None else bias.to(dev),
                          K=K, N=N, KP=int(state["KP"]), aclip=float(state["activation_clip"]), bias_cache={})
        with torch.no_grad():
            self.weight_clip.fill_(float(state["weight_clip"]))
            self.activation_clip.fill_(float(state["activation_clip"]))
        self._attach_head_rotation()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not self.enabled:
            return self.base(x)
        if not x.is_cuda:
            raise RuntimeError("QuantLinear's W4A4 path runs on CUDA tensors only")
        if x.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            raise RuntimeError("x must be bf16, f16 or f32")
        if self._prep is None:
            self.prepare()
        p = self._prep
        K, N = p["K"], p["N"]
        x2 = x.reshape(-1, K)
        if x2.stride(-1) != 1:
            x2 = x2.contiguous()
        bias = None
        if p["bias"] is not None:
            bias = p["bias_cache"].get(x.dtype)
            if bias is None:
                bias = p["bias"].to(x.dtype).contiguous()
                p["bias_cache"][x.dtype] = bias
        M = x2.shape[0]
        if "head_rot" in p:  # per-head Rotation applied to the input online (role 'o')
            if x2.dtype != torch.bfloat16:
                x2 = x2.to(torch.bfloat16)
            hi, lo = p["head_rot"]
            q = ops.rowquant_headrot(x2, hi, lo, "act_sym", clip=p["aclip"])
            y = ops.w4a4_gemm(q.packed, p["packed"], q.scales, p["sw"], M=M, N=N, bias=bias, out_dtype=x.dtype)
        elif self.symmetric and self.int8_activations and M > self.A8_MIN_TOKENS:
            # int8 activation codes straight into the GEMM's TMA (no activation expansion); same bits
            q = ops.rowquant(x2, "act_sym", clip=p["aclip"], rotate=self.rotate, KP=p["KP"], codes=True,
                             packed_out=False)
            y = ops.w4a4_gemm_a8(q.codes, p["packed"], q.scales, p["sw"], M=M, N=N, bias=bias, out_dtype=x.dtype)
        else:
            mode = "act_sym" if self.symmetric else "act_asym_torch"
            q = ops.rowquant(x2, mode, clip=p["aclip"], rotate=self.rotate, KP=p["KP"])
            y = ops.w4a4_gemm(q.packed, p["packed"], q.scales, p["sw"], M=M, N=N,
                              zx=None if self.symmetric else q.zeros, sums=None if self.symmetric else p["wsum"],
                              bias=bias, out_dtype=x.dtype)
        return y.reshape(*x.shape[:-1], N)

    # ------------------------------------------------------------------ shared-input projections
    def quantize_input(self, x2: torch.Tensor) -> "ops.RowQuant":
        """Rotate+quantize a [M, K] input once for several projections that read it (q/k/v, gate/up
        of one layer). Their weights must use the same scheme and K; the result feeds
        forward_quantized of each of them."""
        if self._prep is None:
            self.prepare()
        if "head_rot" in self._prep or not self.symmetric:
            raise NotImplementedError("quantize_input covers the symmetric scheme without online head rotation")
        p = self._prep
        return ops.rowquant(x2, "act_sym", clip=p["aclip"], rotate=self.rotate, KP=p["KP"])

    def forward_quantized(self, q: "ops.RowQuant", M: int, residual: torch.Tensor | None = None,
                          out_dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """This projection on an input already quantised by quantize_input (same K and scheme): the W4A4
        GEMM with the dequant epilogue, plus an optional [M, N] residual added in the epilogue."""
        if self._prep is None:
            self.prepare()
        p = self._prep
        if q.KP != p["KP"]:
            raise ValueError(f"quantised input has KP={q.KP}, this layer expects {p['KP']}")
        bias = None
        if p["bias"] is not None:
            bias = p["bias_cache"].get(out_dtype)
            if bias is None:
                bias = p["bias"].to(out_dtype).contiguous()
                p["bias_cache"][out_dtype] = bias
        return ops.w4a4_gemm(q.packed, p["packed"], q.scales, p["sw"], M=M, N=p["N"], bias=bias, residual=residual,
                             out_dtype=out_dtype)

    def extra_repr(self) -> str:
        return (f"in={self.base.in_features}, out={self.base.out_features}, symmetric={self.symmetric}, "
                f"rotation={self.rotate}, enabled={self.enabled}")
