"""Torch-facing operators over the C ABI (CUDA tensors only).

`quantize` and `matmul` keep the signatures and checks of the reference's
extension (kernel/w4a4.cu:164-230: ``quantize(x, clip, fused)`` and
``matmul(a, b, sx, zx, sw, sums, bias, M, N, fused, force_decode, fp32)``);
`rowquant` and `w4a4_gemm` are the general entry points the W4A4 module uses
(online rotation, symmetric codes, bf16 output, residual).

Outputs are allocated on the input's device, launches go to the current
stream of that device, and everything is asynchronous with respect to the
host (as in the reference). Failures raise RuntimeError (ValueError for int4
codes out of range), mirroring TORCH_CHECK.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib

_DT = {torch.bfloat16: _lib.BF16, torch.float16: _lib.F16, torch.float32: _lib.F32}
_MODES = {"act_sym": _lib.ACT_SYM, "weight_sym": _lib.WEIGHT_SYM, "act_asym": _lib.ACT_ASYM,
          "act_asym_torch": _lib.ACT_ASYM_TORCH}


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(device: torch.device):
    return ctypes.c_void_p(torch.cuda.current_stream(device).cuda_stream)


def _check_cuda(t: torch.Tensor, name: str) -> None:
    if not (t.is_cuda and t.is_contiguous()):
        raise RuntimeError(f"Expected contiguous CUDA tensor for {name}")


# ------------------------------------------------------------------ host helpers
def hadamard(n: int) -> torch.Tensor:
    """+-1 Hadamard matrix of order n (int8, host memory) from the native constructions."""
    out = torch.empty((n, n), dtype=torch.int8)
    _lib.check(_lib.load().dscq_hadamard(n, _ptr(out)), "dscq_hadamard")
    return out


def rotation_split(K: int) -> tuple[int, int]:
    a, b = ctypes.c_int(), ctypes.c_int()
    _lib.check(_lib.load().dscq_rotation_split(K, ctypes.byref(a), ctypes.byref(b)), "dscq_rotation_split")
    return a.value, b.value


_factor_cache: dict = {}


def rotation_factor(K: int, device: torch.device):
    """(a, H_a on `device` or None) for the Kronecker rotation H_a (x) H_(K/a)."""
    key = (K, str(device))
    if key not in _factor_cache:
        a, _ = rotation_split(K)
        _factor_cache[key] = (a, hadamard(a).to(device) if a > 1 else None)
    return _factor_cache[key]


def device_status(device=None, clear: bool = True) -> int:
    """Sticky status bits the kernels raised on `device` (0 = clean). Synchronises the device."""
    dev = torch.device("cuda", torch.cuda.current_device()) if device is None else torch.device(device)
    v = ctypes.c_uint32()
    _lib.check(_lib.load().dscq_device_status(dev.index or 0, ctypes.byref(v), int(clear)), "dscq_device_status")
    return v.value


# ------------------------------------------------------------------ reference-compatible API
def quantize(x: torch.Tensor, clip: float, fused: bool = True):
    """kernel/w4a4.cu:164-187: asymmetric per-row codes; returns [packed, scales, zeros] padded to
    MP = ceil8(M) rows and KP = ceil64(K) columns."""
    _check_cuda(x, "x")
    if x.dtype not in (torch.float16, torch.float32, torch.bfloat16):
        raise RuntimeError("Only FP16, BF16 and FP32 inputs are supported")
    if not (x.dim() == 2 and 0 < x.size(0) <= 65535 and 0 < x.size(1) <= 1048576):
        raise RuntimeError("Require 1<=M<=65535 and 1<=K<=1048576")
    if not (0.5 <= clip <= 1.0):
        raise RuntimeError("Activation clip must be in [0.5,1]")
    M, K = x.shape
    MP, KP = (M + 7) // 8 * 8, (K + 63) // 64 * 64
    with torch.cuda.device(x.device):
        packed = torch.empty((MP, KP // 2), dtype=torch.uint8, device=x.device)
        scales = torch.empty((MP,), dtype=torch.float32, device=x.device)
        zeros = torch.empty((MP,), dtype=torch.int32, device=x.device)
        rc = _lib.load().dscq_quantize(_ptr(x), _DT[x.dtype], M, K, float(clip), int(bool(fused)), _ptr(packed),
                                       _ptr(scales), _ptr(zeros), _stream(x.device))
    _lib.check(rc, "quantize")
    return [packed, scales, zeros]


def matmul(a, b, sx, zx, sw, sums, bias, M: int, N: int, fused: bool = True, force_decode: bool = False,
           fp32: bool = False, *, out_dtype: torch.dtype | None = None, residual: torch.Tensor | None = None):
    """kernel/w4a4.cu:189-225. Returns [out [M, N], raw [M, N] int32 (or empty when fused)].
    out dtype is float32 if `fp32` else float16, unless `out_dtype` overrides it (bf16)."""
    for name, t in (("a", a), ("b", b), ("sx", sx), ("zx", zx), ("sw", sw), ("sums", sums), ("bias", bias)):
        _check_cuda(t, name)
        if t.device != a.device:
            raise RuntimeError("All buffers must be on the same device")
    if not (a.dim() == 2 and b.dim() == 2 and a.dtype == torch.uint8 and b.dtype == torch.uint8):
        raise RuntimeError("Packed operands must be byte matrices")
    KP, MP, NP = a.size(1) * 2, (M + 7) // 8 * 8, (N + 7) // 8 * 8
    if not (0 < M <= 65535 and N > 0 and 0 < KP <= 1048576 and KP % 64 == 0):
        raise RuntimeError("Invalid dimensions")
    if not (a.size(0) >= MP and b.size(0) >= NP and b.size(1) == a.size(1)):
        raise RuntimeError("Invalid padded operand shapes")
    if not (sx.dtype == torch.float32 and sw.dtype == torch.float32 and zx.dtype == torch.int32
            and sums.dtype == torch.int32):
        raise RuntimeError("Invalid metadata dtypes")
    if not (sx.numel() >= MP and zx.numel() >= MP and sw.numel() >= NP and sums.numel() >= NP):
        raise RuntimeError("Metadata too short")
    dtype = out_dtype if out_dtype is not None else (torch.float32 if fp32 else torch.float16)
    if not (bias.dtype == dtype and (bias.numel() == 0 or bias.numel() == N)):
        raise RuntimeError("Bias shape/dtype mismatch")
    with torch.cuda.device(a.device):
        out = torch.empty((M, N), dtype=dtype, device=a.device)
        raw = (torch.empty((0,), dtype=torch.int32, device=a.device) if fused
               else torch.empty((M, N), dtype=torch.int32, device=a.device))
        if residual is not None:
            _check_cuda(residual, "residual")
            if residual.shape != (M, N) or residual.dtype != dtype:
                raise RuntimeError("Residual shape/dtype mismatch")
        variant = _lib.GEMM_SMALL_M if force_decode else _lib.GEMM_AUTO
        rc = _lib.load().dscq_matmul(_ptr(a), _ptr(b), _ptr(sx), _ptr(zx), _ptr(sw), _ptr(sums),
                                     _ptr(bias) if bias.numel() else None, _ptr(residual), M, N, KP, _DT[dtype],
                                     _ptr(out), None if fused else _ptr(raw), variant, _stream(a.device))
    _lib.check(rc, "matmul")
    return [out, raw]


# ------------------------------------------------------------------ W4A4 path entry points
@dataclass
class RowQuant:
    packed: torch.Tensor        # [rows_out, KP/2] u8
    scales: torch.Tensor        # [rows_out] f32
    zeros: torch.Tensor | None  # [rows_out] i32 (asymmetric modes)
    row_sums: torch.Tensor | None
    codes: torch.Tensor | None  # [rows_out, KP] int8
    KP: int


def rowquant(x: torch.Tensor, mode: str = "act_sym", clip: float = 1.0, rotate: bool = False,
             rows_out: int | None = None, KP: int | None = None, codes: bool = False,
             row_sums: bool = False, variant: str = "auto", packed_out: bool = True) -> RowQuant:
    """Per-row int4 quantisation of a 2-D CUDA tensor with an optional online Hadamard rotation
    (y = x (H_a (x) H_b) / sqrt(K)), one fused kernel. See include/dscq_b200.h (dscq_rowquant).
    `variant`: "auto", "tc" (tcgen05 kernel) or "legacy" (CUDA-core kernels), for A/B timing.
    `packed_out=False` (with codes=True) writes only the int8 codes, the A operand of w4a4_gemm_a8."""
    if not x.is_cuda:
        raise RuntimeError("rowquant runs on CUDA tensors only")
    if x.dim() != 2 or x.stride(1) != 1:
        raise RuntimeError("rowquant expects a 2-D tensor with unit column stride")
    if x.dtype not in _DT:
        raise RuntimeError("x must be bf16, f16 or f32")
    M, K = x.shape
    rows_out = M if rows_out is None else rows_out
    KP = (K + 63) // 64 * 64 if KP is None else KP
    m = _MODES[mode]
    asym = m in (_lib.ACT_ASYM, _lib.ACT_ASYM_TORCH)
    dev = x.device
    with torch.cuda.device(dev):
        if not packed_out and not codes:
            raise ValueError("rowquant needs packed_out or codes")
        packed = torch.empty((rows_out, KP // 2), dtype=torch.uint8, device=dev) if packed_out else None
        scales = torch.empty((rows_out,), dtype=torch.float32, device=dev)
        zeros = torch.empty((rows_out,), dtype=torch.int32, device=dev) if asym else None
        sums = torch.empty((rows_out,), dtype=torch.int32, device=dev) if row_sums else None
        cds = torch.empty((rows_out, KP), dtype=torch.int8, device=dev) if codes else None
        a, h = rotation_factor(K, dev) if rotate else (1, None)
        var = {"auto": _lib.QUANT_AUTO, "tc": _lib.QUANT_TC, "legacy": _lib.QUANT_LEGACY}[variant]
        rc = _lib.load().dscq_rowquant_variant(_ptr(x), _DT[x.dtype], M, K, x.stride(0), int(rotate), a, _ptr(h), m,
                                               float(clip), rows_out, KP, _ptr(packed), KP // 2 if packed_out else 0,
                                               _ptr(scales),
                                               _ptr(zeros), _ptr(sums), _ptr(cds), KP if codes else 0, var,
                                               _stream(dev))
    _lib.check(rc, "rowquant")
    return RowQuant(packed, scales, zeros, sums, cds, KP)


def head_rotation_operands(R: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Per-head rotation matrices R [heads, 128, 128] (fp32, e.g. core/transforms.py Rotation.matrices())
    -> the (hi, lo) bf16 operands of rowquant_headrot: hi + lo ~ R to ~2^-17, each stored transposed per
    head (op[h][e][d] = R[h][d][e]). Call once per set of matrices."""
    if R.dim() != 3 or R.shape[1:] != (128, 128):
        raise ValueError("R must be [heads, 128, 128]")
    if not R.is_cuda:
        raise RuntimeError("R must be a CUDA tensor")
    Rt = R.detach().float().transpose(1, 2).contiguous()
    hi = Rt.to(torch.bfloat16)
    lo = (Rt - hi.float()).to(torch.bfloat16)
    return hi.contiguous(), lo.contiguous()


def rowquant_headrot(x: torch.Tensor, hi: torch.Tensor, lo: torch.Tensor, mode: str = "act_sym", clip: float = 1.0,
                     rows_out: int | None = None, codes: bool = False, packed_out: bool = True) -> RowQuant:
    """Online per-head block rotation (y = x blockdiag(R_h)) fused with symmetric per-row int4 quantisation,
    one tcgen05 kernel (include/dscq_b200.h, dscq_rowquant_headrot). x [M, 128 * heads] bf16; hi, lo from
    head_rotation_operands."""
    if not x.is_cuda or x.dtype != torch.bfloat16 or x.dim() != 2 or x.stride(1) != 1:
        raise RuntimeError("rowquant_headrot expects a 2-D bf16 CUDA tensor with unit column stride")
    M, K = x.shape
    heads = hi.shape[0]
    if K != 128 * heads or hi.shape != lo.shape:
        raise ValueError("x must have 128 * heads columns")
    rows_out = M if rows_out is None else rows_out
    m = _MODES[mode]
    dev = x.device
    with torch.cuda.device(dev):
        packed = torch.empty((rows_out, K // 2), dtype=torch.uint8, device=dev) if packed_out else None
        scales = torch.empty((rows_out,), dtype=torch.float32, device=dev)
        cds = torch.empty((rows_out, K), dtype=torch.int8, device=dev) if codes else None
        rc = _lib.load().dscq_rowquant_headrot(_ptr(x), M, K, x.stride(0), heads, _ptr(hi), _ptr(lo), m, float(clip),
                                               rows_out, K, _ptr(packed), K // 2 if packed_out else 0, _ptr(scales),
                                               _ptr(cds), K if codes else 0, _stream(dev))
    _lib.check(rc, "rowquant_headrot")
    return RowQuant(packed, scales, None, None, cds, K)


def _check_gemm_metadata(dev: torch.device, M: int, N: int, out_dtype: torch.dtype, sx, sw, zx=None, sums=None,
                         bias=None, residual=None) -> None:
    """Argument checks shared by the GEMM entry points (the same checks as the reference's matmul,
    kernel/w4a4.cu:192-202): the kernels read sx[0..M), sw / sums / bias [0..N), zx [0..M) and
    residual [M, N] through raw pointers, so a short, mistyped or misplaced tensor is rejected here."""
    if out_dtype not in _DT:
        raise RuntimeError("out_dtype must be bf16, f16 or f32")
    for name, t, dtype, n in (("sx", sx, torch.float32, M), ("sw", sw, torch.float32, N), ("zx", zx, torch.int32, M),
                              ("sums", sums, torch.int32, N)):
        if t is None:
            continue
        if not t.is_cuda or t.device != dev:
            raise RuntimeError(f"{name} must be a CUDA tensor on {dev}")
        if t.dtype != dtype:
            raise RuntimeError(f"{name} must be {dtype}")
        if not t.is_contiguous() or t.numel() < n:
            raise RuntimeError(f"{name} must be contiguous with at least {n} elements")
    if (zx is None) != (sums is None):
        raise RuntimeError("zx and sums go together (asymmetric activations)")
    if bias is not None:
        if not bias.is_cuda or bias.device != dev or bias.dtype != out_dtype:
            raise RuntimeError(f"bias must be a {out_dtype} CUDA tensor on {dev} (the output dtype)")
        if not bias.is_contiguous() or bias.numel() != N:
            raise RuntimeError(f"bias must be contiguous with N={N} elements")
    if residual is not None:
        if not residual.is_cuda or residual.device != dev or residual.dtype != out_dtype:
            raise RuntimeError(f"residual must be a {out_dtype} CUDA tensor on {dev} (the output dtype)")
        if tuple(residual.shape) != (M, N) or not residual.is_contiguous():
            raise RuntimeError(f"residual must be a contiguous [{M}, {N}] tensor")


def w4a4_gemm(a: torch.Tensor, b: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, *, M: int | None = None,
              N: int | None = None, zx: torch.Tensor | None = None, sums: torch.Tensor | None = None,
              bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
              out_dtype: torch.dtype = torch.bfloat16, return_raw: bool = False, want_out: bool = True,
              variant: str = "auto"):
    """out[m, n] = ((sum_k a[m,k] b[n,k] + (8 - zx[m]) sums[n]) * sx[m]) * sw[n] + bias[n] + residual[m, n]
    on packed int4 operands (tcgen05 int8 GEMM). Returns out, or (out, raw) with return_raw.
    a [>= M, KP/2] and b [>= N, KP/2] are contiguous u8 rows; M and N default to their row counts."""
    for name, t in (("a", a), ("b", b)):
        _check_cuda(t, name)
        if t.dtype != torch.uint8 or t.dim() != 2:
            raise RuntimeError(f"{name} must be a 2-D uint8 tensor of packed int4 codes")
    dev = a.device
    if b.device != dev:
        raise RuntimeError("a and b must be on the same device")
    M = a.size(0) if M is None else int(M)
    N = b.size(0) if N is None else int(N)
    KP = a.size(1) * 2
    if b.size(1) != a.size(1):
        raise RuntimeError("a and b must have the same packed K")
    if not (0 < M <= a.size(0) and 0 < N <= b.size(0)):
        raise RuntimeError(f"need 0 < M <= a.size(0) and 0 < N <= b.size(0) (M={M}, N={N})")
    _check_gemm_metadata(dev, M, N, out_dtype, sx, sw, zx, sums, bias, residual)
    with torch.cuda.device(dev):
        out = torch.empty((M, N), dtype=out_dtype, device=dev) if want_out else None
        raw = torch.empty((M, N), dtype=torch.int32, device=dev) if return_raw else None
        v = {"auto": _lib.GEMM_AUTO, "small_m": _lib.GEMM_SMALL_M, "large_m": _lib.GEMM_LARGE_M,
             "large_m_direct": _lib.GEMM_LARGE_M_DIRECT, "large_m_pair": _lib.GEMM_LARGE_M_PAIR,
             "small_m_tc": _lib.GEMM_SMALL_M_TC, "large_m_pair_tmem": _lib.GEMM_LARGE_M_PAIR_TMEM}[variant]
        rc = _lib.load().dscq_matmul(_ptr(a), _ptr(b), _ptr(sx), _ptr(zx), _ptr(sw), _ptr(sums), _ptr(bias),
                                     _ptr(residual), M, N, KP, _DT[out_dtype], _ptr(out), _ptr(raw), v, _stream(dev))
    _lib.check(rc, "w4a4_gemm")
    return (out, raw) if return_raw else out


def w4a4_gemm_a8(a: torch.Tensor, b: torch.Tensor, sx: torch.Tensor, sw: torch.Tensor, *, M: int | None = None,
                 N: int | None = None, bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                 out_dtype: torch.dtype = torch.bfloat16, return_raw: bool = False, variant: str = "auto"):
    """w4a4_gemm with int8 activation codes a [M, KP] (values in [-8, 7], e.g. rowquant(..., codes=True,
    packed_out=False)) and packed int4 weights b [N, KP/2]; symmetric activations only. Same bits as
    w4a4_gemm on the packed form of a. `variant`: "auto" (CTA pairs for 256-wide tiles), "large_m"
    (1-CTA kernel) or "large_m_pair" (CTA pairs)."""
    _check_cuda(b, "b")
    if b.dtype != torch.uint8 or b.dim() != 2:
        raise RuntimeError("b must be a 2-D uint8 tensor of packed int4 codes")
    KP = b.size(1) * 2
    if not a.is_cuda or a.dtype != torch.int8 or a.dim() != 2 or a.stride(1) != 1 or a.size(1) < KP:
        raise RuntimeError("a must be CUDA int8 codes [M, >= KP] with unit column stride")
    dev = a.device
    if b.device != dev:
        raise RuntimeError("a and b must be on the same device")
    M = a.size(0) if M is None else int(M)
    N = b.size(0) if N is None else int(N)
    if not (0 < M <= a.size(0) and 0 < N <= b.size(0)):
        raise RuntimeError(f"need 0 < M <= a.size(0) and 0 < N <= b.size(0) (M={M}, N={N})")
    _check_gemm_metadata(dev, M, N, out_dtype, sx, sw, None, None, bias, residual)
    with torch.cuda.device(dev):
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
        raw = torch.empty((M, N), dtype=torch.int32, device=dev) if return_raw else None
        v = {"auto": _lib.GEMM_AUTO, "large_m": _lib.GEMM_LARGE_M, "large_m_pair": _lib.GEMM_LARGE_M_PAIR}[variant]
        rc = _lib.load().dscq_matmul_a8_variant(_ptr(a), a.stride(0), _ptr(b), _ptr(sx), _ptr(sw), _ptr(bias),
                                                _ptr(residual), M, N, KP, _DT[out_dtype], _ptr(out), _ptr(raw), v,
                                                _stream(dev))
    _lib.check(rc, "matmul_a8")
    return (out, raw) if return_raw else out


def pack_int4_cuda(codes: torch.Tensor) -> torch.Tensor:
    """core/quantization.py:31-40 on the GPU (ValueError for ndim != 2 or codes outside [-8, 7])."""
    if codes.ndim != 2:
        raise ValueError("Packed weights must be a matrix.")
    if not codes.is_cuda:
        raise RuntimeError("pack_int4 runs on CUDA tensors only")
    # same order as the reference: convert to int8 first, then range-check the int8 values
    c = codes.to(torch.int8).contiguous()
    rows, K = c.shape
    with torch.cuda.device(c.device):
        packed = torch.empty((rows, (K + 1) // 2), dtype=torch.uint8, device=c.device)
        bad = torch.zeros((1,), dtype=torch.int32, device=c.device)
        if rows and K:
            rc = _lib.load().dscq_pack_int4(_ptr(c), rows, K, K, _ptr(packed), (K + 1) // 2, _ptr(bad),
                                            _stream(c.device))
            _lib.check(rc, "pack_int4")
    if int(bad.item()):
        raise ValueError("Signed INT4 code out of range.")
    return packed


def unpack_int4_cuda(packed: torch.Tensor, width: int) -> torch.Tensor:
    """core/quantization.py:42-45 on the GPU."""
    if not packed.is_cuda:
        raise RuntimeError("unpack_int4 runs on CUDA tensors only")
    p = packed.contiguous()
    rows = p.size(0)
    w = min(width, p.size(1) * 2)
    with torch.cuda.device(p.device):
        codes = torch.empty((rows, w), dtype=torch.int8, device=p.device)
        if rows and w:
            rc = _lib.load().dscq_unpack_int4(_ptr(p), rows, p.size(1), w, _ptr(codes), w, _stream(p.device))
            _lib.check(rc, "unpack_int4")
    return codes


# ------------------------------------------------------------------ prefill element-wise operators
def _bf16_cuda(t: torch.Tensor, name: str) -> None:
    if not (t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous()):
        raise RuntimeError(f"{name} must be a contiguous bf16 CUDA tensor")


def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float) -> torch.Tensor:
    """bf16(bf16(x * rsqrt(mean(x^2, -1) + eps)) * w) over the last dimension, one kernel."""
    _bf16_cuda(x, "x")
    _bf16_cuda(w, "w")
    H = x.shape[-1]
    if w.numel() != H:
        raise RuntimeError("w must have the last dimension of x")
    y = torch.empty_like(x)
    _lib.check(_lib.load().dscq_rmsnorm(_ptr(x), _ptr(w), x.numel() // H, H, float(eps), _ptr(y), _stream(x.device)),
               "rmsnorm")
    return y


def rope_(q: torch.Tensor, k: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> None:
    """Rotary embeddings (rotate-half form) in place on q [S, Hq, D] and k [S, Hk, D]; cos / sin [S, D]."""
    for name, t in (("q", q), ("k", k), ("cos", cos), ("sin", sin)):
        _bf16_cuda(t, name)
    S, Hq, D = q.shape
    if k.shape[0] != S or k.shape[2] != D or cos.shape != (S, D) or sin.shape != (S, D):
        raise RuntimeError("rope shapes: q [S, Hq, D], k [S, Hk, D], cos / sin [S, D]")
    _lib.check(_lib.load().dscq_rope(_ptr(q), _ptr(k), _ptr(cos), _ptr(sin), S, Hq, k.shape[1], D, _stream(q.device)),
               "rope")


def silu_mul(g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
    """bf16(bf16(silu(g)) * u), one kernel."""
    _bf16_cuda(g, "g")
    _bf16_cuda(u, "u")
    if g.shape != u.shape:
        raise RuntimeError("g and u must have the same shape")
    y = torch.empty_like(g)
    _lib.check(_lib.load().dscq_silu_mul(_ptr(g), _ptr(u), g.numel(), _ptr(y), _stream(g.device)), "silu_mul")
    return y
