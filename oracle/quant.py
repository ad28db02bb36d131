"""Oracle quantisation math (numpy restatement).  TEST INFRASTRUCTURE ONLY.

Restates the reference's fake quantisation, ``intent_quant.py:221-312``
(``_absmax_scale`` and ``fake_quantize_tensor``), step by step in float32 so
that integer codes and reconstructions are bit-identical to the reference's
torch CPU arithmetic:

* scale  = max(absmax / 127, 1e-8), absmax reduced over the scale span
  (``intent_quant.py:221-226``; the reference reduces over every axis but the
  last, i.e. one scale per channel for the whole block);
* INT8 / INT4: ``round_half_even(clamp(x / scale, -q, q))`` with q = 127 / 7
  and the SAME /127 scale for both (``intent_quant.py:260-280``);
* FP8: ``e4m3fn(x / scale) * scale`` (``intent_quant.py:241-258``);
* INT4_RESIDUAL: INT4 base, then the residual re-scaled by its own absmax/127
  and clamped to +-7 (``intent_quant.py:282-307``);
* FP16: ``x.half()``; SKIP: zeros (``intent_quant.py:238-239, 309-310``).

The page-level helpers apply the same formulas with a different reduction span
(per page, per 32-channel group, or per channel), which is what the paged kernels
consume.  The packed INT4 layout defined here (``int4_d_index``) is the storage
format of this project's INT4 / INT4_RESIDUAL page pools.
"""

from __future__ import annotations

from typing import Dict, Optional, Sequence, Tuple

import numpy as np

F32 = np.float32
PRECISIONS = ("FP16", "FP8", "INT8", "INT4", "INT4_RESIDUAL", "SKIP")


# --------------------------------------------------------------------------- #
#  e4m3fn (OCP FP8, "fn" = finite, NaN only) encode / decode, round-half-even
# --------------------------------------------------------------------------- #

def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """float32 -> e4m3fn codes (uint8), round-to-nearest-even.

    Matches torch's ``Tensor.to(torch.float8_e4m3fn)``: magnitudes that round
    above 448 become NaN (0x7F | sign), subnormals are m * 2**-9.
    """
    x = np.asarray(x, dtype=np.float32).astype(np.float64)
    sign = (np.signbit(x)).astype(np.uint8) << 7
    a = np.abs(x)
    code = np.zeros(a.shape, dtype=np.int64)
    # normal range: a >= 2**-6
    normal = a >= 2.0 ** -6
    m, e = np.frexp(np.where(normal, a, 1.0))  # a = m * 2**e, m in [0.5, 1)
    e = e - 1                                   # a = (2m) * 2**e, 2m in [1, 2)
    frac = (2.0 * m - 1.0) * 8.0                # exact in float64
    q = np.rint(frac).astype(np.int64)          # half-to-even
    carry = q >= 8
    q = np.where(carry, 0, q)
    e = np.where(carry, e + 1, e)
    exp_field = e + 7
    normal_code = (exp_field << 3) | q
    # subnormal: value = k * 2**-9, k in 0..8 (k == 8 is the smallest normal)
    k = np.rint(a / 2.0 ** -9).astype(np.int64)
    code = np.where(normal, normal_code, k)
    nan = (code > 0x7E) | np.isnan(a)
    code = np.where(nan, 0x7F, code)
    return (code.astype(np.uint8) | sign).astype(np.uint8)


def e4m3_to_f32(code: np.ndarray) -> np.ndarray:
    """e4m3fn codes (uint8) -> float32 (exact)."""
    c = np.asarray(code, dtype=np.uint8).astype(np.int64)
    s = np.where(c & 0x80, -1.0, 1.0)
    ef = (c >> 3) & 0xF
    mf = c & 0x7
    val = np.where(ef == 0, mf * 2.0 ** -9, (1.0 + mf / 8.0) * np.exp2(ef - 7.0))
    val = np.where((c & 0x7F) == 0x7F, np.nan, val)
    return (s * val).astype(np.float32)


# --------------------------------------------------------------------------- #
#  Reference-granularity fake quantisation (intent_quant.py:221-312)
# --------------------------------------------------------------------------- #

def absmax_scale(x: np.ndarray, axes: Optional[Sequence[int]] = None) -> Tuple[np.ndarray, np.ndarray]:
    """Symmetric absmax scale, ``intent_quant.py:221-226``.

    ``axes=None`` reduces over every axis but the last (the reference's
    per-channel rule).  Returns ``(scale, absmax)`` with keepdims.
    """
    x = np.asarray(x, dtype=F32)
    if axes is None:
        axes = tuple(range(x.ndim - 1))
    absmax = np.abs(x).max(axis=tuple(axes), keepdims=True).astype(F32)
    scale = (absmax / F32(127.0)).astype(F32)
    scale = np.maximum(scale, F32(1e-8)).astype(F32)
    return scale, absmax


def _int_codes(x: np.ndarray, scale: np.ndarray, max_q: int) -> np.ndarray:
    y = (x / scale).astype(F32)
    y = np.clip(y, F32(-max_q), F32(max_q))
    return np.rint(y).astype(np.int8)


def fake_quantize(x: np.ndarray, precision: str, axes: Optional[Sequence[int]] = None) -> Dict[str, np.ndarray]:
    """Fake-quantise ``x`` (float32) like ``fake_quantize_tensor``.

    Returns a dict with ``recon`` (float32), and per precision the integer /
    fp8 ``codes``, ``scale`` and (INT4_RESIDUAL) ``res_codes`` / ``res_scale``.
    ``axes`` selects the scale span (default: the reference's per-channel span).
    """
    x = np.asarray(x, dtype=F32)
    p = precision.upper()
    if p == "FP16":
        return {"recon": x.astype(np.float16).astype(F32)}
    if p == "SKIP":
        return {"recon": np.zeros_like(x)}
    scale, _ = absmax_scale(x, axes)
    if p == "FP8":
        codes = f32_to_e4m3((x / scale).astype(F32))
        recon = (e4m3_to_f32(codes) * scale).astype(F32)
        return {"recon": recon, "codes": codes, "scale": scale}
    if p in ("INT8", "INT4"):
        max_q = 127 if p == "INT8" else 7
        codes = _int_codes(x, scale, max_q)
        recon = (codes.astype(F32) * scale).astype(F32)
        return {"recon": recon, "codes": codes, "scale": scale}
    if p == "INT4_RESIDUAL":
        codes = _int_codes(x, scale, 7)
        base = (codes.astype(F32) * scale).astype(F32)
        residual = (x - base).astype(F32)
        res_scale, _ = absmax_scale(residual, axes)
        res_codes = _int_codes(residual, res_scale, 7)
        res_recon = (res_codes.astype(F32) * res_scale).astype(F32)
        recon = (base + res_recon).astype(F32)
        return {"recon": recon, "codes": codes, "scale": scale,
                "res_codes": res_codes, "res_scale": res_scale}
    raise ValueError(f"Unknown precision: {precision}")


# --------------------------------------------------------------------------- #
#  Page-granularity quantisation (the formats the paged kernels read)
# --------------------------------------------------------------------------- #

SCALE_MODES = ("page", "group32", "channel")


def n_scales(scale_mode: str, head_dim: int) -> int:
    if scale_mode == "page":
        return 1
    if scale_mode == "group32":
        return head_dim // 32
    if scale_mode == "channel":
        return head_dim
    raise ValueError(scale_mode)


def expand_scales(scales: np.ndarray, scale_mode: str, head_dim: int) -> np.ndarray:
    """[P, n_scales] -> [P, 1, D] broadcastable per-channel scales."""
    scales = np.asarray(scales, dtype=F32)
    if scale_mode == "page":
        out = np.repeat(scales, head_dim, axis=1)
    elif scale_mode == "group32":
        out = np.repeat(scales, 32, axis=1)
    else:
        out = scales
    return out[:, None, :].astype(F32)


def page_scales(x: np.ndarray, scale_mode: str) -> np.ndarray:
    """Per-page scale array [P, n_scales] with the reference's formula."""
    x = np.asarray(x, dtype=F32)
    P, PS, D = x.shape
    a = np.abs(x)
    if scale_mode == "page":
        absmax = a.reshape(P, -1).max(axis=1, keepdims=True)
    elif scale_mode == "group32":
        absmax = a.reshape(P, PS, D // 32, 32).max(axis=(1, 3))
    elif scale_mode == "channel":
        absmax = a.max(axis=1)
    else:
        raise ValueError(scale_mode)
    scale = (absmax.astype(F32) / F32(127.0)).astype(F32)
    return np.maximum(scale, F32(1e-8)).astype(F32)


def quantize_pages(x: np.ndarray, precision: str, scale_mode: str = "page",
                   scales: Optional[np.ndarray] = None,
                   res_scales: Optional[np.ndarray] = None) -> Dict[str, np.ndarray]:
    """Quantise pages ``x`` [P, PS, D] (float32) into one page format.

    Same arithmetic as ``fake_quantize`` with a per-page scale span.  Optional
    ``scales`` / ``res_scales`` ([P, n_scales]) replace the computed ones, which
    lets a caller use spans wider than one page (e.g. the reference's
    per-block-per-channel scale replicated onto each page of the block).
    Returns ``codes`` (int8 values, or uint8 e4m3 codes), ``scale``
    [P, n_scales], ``recon`` float32, plus ``res_codes``/``res_scale`` for
    INT4_RESIDUAL.
    """
    x = np.asarray(x, dtype=F32)
    P, PS, D = x.shape
    p = precision.upper()
    if p == "FP16":
        return {"codes": x.astype(np.float16), "recon": x.astype(np.float16).astype(F32)}
    if p == "SKIP":
        return {"recon": np.zeros_like(x)}
    s = page_scales(x, scale_mode) if scales is None else np.asarray(scales, dtype=F32)
    se = expand_scales(s, scale_mode, D)
    if p == "FP8":
        codes = f32_to_e4m3((x / se).astype(F32))
        return {"codes": codes, "scale": s, "recon": (e4m3_to_f32(codes) * se).astype(F32)}
    if p in ("INT8", "INT4"):
        codes = _int_codes(x, se, 127 if p == "INT8" else 7)
        return {"codes": codes, "scale": s, "recon": (codes.astype(F32) * se).astype(F32)}
    if p == "INT4_RESIDUAL":
        codes = _int_codes(x, se, 7)
        base = (codes.astype(F32) * se).astype(F32)
        residual = (x - base).astype(F32)
        rs = page_scales(residual, scale_mode) if res_scales is None else np.asarray(res_scales, dtype=F32)
        rse = expand_scales(rs, scale_mode, D)
        res_codes = _int_codes(residual, rse, 7)
        recon = (base + (res_codes.astype(F32) * rse).astype(F32)).astype(F32)
        return {"codes": codes, "scale": s, "res_codes": res_codes, "res_scale": rs, "recon": recon}
    raise ValueError(f"Unknown precision: {precision}")


def dequantize_pages(codes: np.ndarray, precision: str, scale_mode: str, scale: np.ndarray,
                     res_codes: Optional[np.ndarray] = None,
                     res_scale: Optional[np.ndarray] = None) -> np.ndarray:
    """Inverse of ``quantize_pages`` (float32 reconstruction)."""
    p = precision.upper()
    codes = np.asarray(codes)
    D = codes.shape[-1]
    if p == "FP16":
        return codes.astype(F32)
    se = expand_scales(scale, scale_mode, D)
    if p == "FP8":
        return (e4m3_to_f32(codes) * se).astype(F32)
    base = (codes.astype(F32) * se).astype(F32)
    if p in ("INT8", "INT4"):
        return base
    if p == "INT4_RESIDUAL":
        rse = expand_scales(res_scale, scale_mode, D)
        return (base + (np.asarray(res_codes).astype(F32) * rse).astype(F32)).astype(F32)
    raise ValueError(precision)


# --------------------------------------------------------------------------- #
#  Packed INT4 storage layout
# --------------------------------------------------------------------------- #

# Nibble n of 32-bit word w (bits 4n..4n+3, little-endian bytes) of a packed
# row holds the code of channel d = 32*(w//4) + 4*(w%4) + INT4_NIBBLE_OFFSET[n].
# Values are stored offset-binary (code + 8).  The pairing (n, n+4) -> (d, d+1)
# lets one masked 32-bit op expose two consecutive channels as a half2.
INT4_NIBBLE_OFFSET = (0, 2, 16, 18, 1, 3, 17, 19)


def int4_d_index(head_dim: int) -> np.ndarray:
    """[head_dim // 8, 8] array: channel held by (word, nibble)."""
    if head_dim % 32:
        raise ValueError("INT4 pages need head_dim % 32 == 0")
    w = np.arange(head_dim // 8)
    d0 = 32 * (w // 4) + 4 * (w % 4)
    return d0[:, None] + np.asarray(INT4_NIBBLE_OFFSET)[None, :]


def pack_int4(codes: np.ndarray) -> np.ndarray:
    """int codes in [-8, 7], shape [..., D] -> uint8 [..., D // 2]."""
    codes = np.asarray(codes).astype(np.int64)
    D = codes.shape[-1]
    idx = int4_d_index(D)
    u = (codes + 8).astype(np.uint64)
    words = np.zeros(codes.shape[:-1] + (D // 8,), dtype=np.uint64)
    for n in range(8):
        words |= u[..., idx[:, n]] << np.uint64(4 * n)
    return words.astype("<u4").view(np.uint8).reshape(codes.shape[:-1] + (D // 2,))


def unpack_int4(packed: np.ndarray) -> np.ndarray:
    """uint8 [..., D // 2] -> int8 codes [..., D]."""
    packed = np.ascontiguousarray(np.asarray(packed, dtype=np.uint8))
    D = packed.shape[-1] * 2
    words = packed.view("<u4").astype(np.int64)
    idx = int4_d_index(D)
    out = np.zeros(packed.shape[:-1] + (D,), dtype=np.int8)
    for n in range(8):
        out[..., idx[:, n]] = (((words >> (4 * n)) & 0xF) - 8).astype(np.int8)
    return out
