"""Python side of the attention entry points (include/zlift_attention.h).

``FlashParams`` / ``FmhaParams`` are ctypes images of the two parameter
blocks the reference decodes (zblas/zblas_gpu.cpp:695-739, :755-784).
``flash_forward`` fills a FlashAttention-2 block from tensors laid out
[batch, seq, heads, dim] (strides taken from the tensors) and calls
``zlift_flash_fwd`` on the given stream.
"""
from __future__ import annotations

import ctypes
import math

from . import load

c_vp, c_ll, c_int, c_float, c_ub = (ctypes.c_void_p, ctypes.c_longlong, ctypes.c_int,
                                    ctypes.c_float, ctypes.c_ubyte)


class FlashParams(ctypes.Structure):
    _fields_ = [
        ("q_ptr", c_vp), ("k_ptr", c_vp), ("v_ptr", c_vp),
        ("q_batch_stride", c_ll), ("k_batch_stride", c_ll), ("v_batch_stride", c_ll),
        ("q_row_stride", c_ll), ("k_row_stride", c_ll), ("v_row_stride", c_ll),
        ("q_head_stride", c_ll), ("k_head_stride", c_ll), ("v_head_stride", c_ll),
        ("h", c_int), ("h_k", c_int), ("h_h_k_ratio", c_int),
        ("o_ptr", c_vp), ("oaccum_ptr", c_vp),
        ("o_batch_stride", c_ll), ("o_row_stride", c_ll), ("o_head_stride", c_ll),
        ("p_ptr", c_vp),
        ("softmax_lse_ptr", c_vp), ("softmax_lseaccum_ptr", c_vp),
        ("b", c_int), ("seqlen_q", c_int), ("seqlen_k", c_int), ("seqlen_knew", c_int),
        ("d", c_int), ("seqlen_q_rounded", c_int), ("seqlen_k_rounded", c_int),
        ("d_rounded", c_int), ("rotary_dim", c_int), ("total_q", c_int),
        ("scale_softmax", c_float), ("scale_softmax_log2", c_float),
        ("opaque", c_ub * 148),
        ("p_dropout", c_float), ("p_dropout_in_uint8_t", c_ub),
        ("rp_dropout", c_float), ("scale_softmax_rp_dropout", c_float),
        ("window_size_left", c_int), ("window_size_right", c_int),
    ]


class FlashBlock(ctypes.Structure):
    """The 448 bytes the flash entry receives: the parameters, zero padding,
    then is_bf16 (byte 440) and is_causal (byte 441)."""
    _fields_ = [("p", FlashParams), ("pad", c_ub * (440 - ctypes.sizeof(FlashParams))),
                ("is_bf16", c_ub), ("is_causal", c_ub), ("tail", c_ub * 6)]


class FmhaParams(ctypes.Structure):
    _fields_ = [
        ("query_ptr", c_vp), ("key_ptr", c_vp), ("value_ptr", c_vp), ("attn_bias_ptr", c_vp),
        ("seqstart_q_ptr", c_vp), ("seqstart_k_ptr", c_vp), ("seqlen_k_ptr", c_vp),
        ("causal_diagonal_offset", ctypes.c_uint),
        ("output_ptr", c_vp), ("output_accum_ptr", c_vp), ("logsumexp_ptr", c_vp),
        ("window_size", c_int), ("scale", c_float),
        ("head_dim", c_int), ("head_dim_value", c_int), ("num_queries", c_int),
        ("num_keys", c_int), ("num_keys_absolute", c_int),
        ("custom_mask_type", c_ub),
        ("q_strideM", c_int), ("k_strideM", c_int), ("v_strideM", c_int),
        ("bias_strideM", c_int), ("o_strideM", c_int),
        ("q_strideH", c_int), ("k_strideH", c_int), ("v_strideH", c_int),
        ("bias_strideH", c_ll),
        ("q_strideB", c_ll), ("k_strideB", c_ll), ("v_strideB", c_ll), ("bias_strideB", c_ll),
        ("num_batches", c_int), ("num_heads", c_int),
        ("use_dropout", c_ub),
    ]


assert ctypes.sizeof(FlashBlock) == 448
assert FlashParams.softmax_lse_ptr.offset == 160 and FlashParams.window_size_left.offset == 388
assert FmhaParams.num_batches.offset == 192 and FmhaParams.custom_mask_type.offset == 116


def _elem(t) -> int:
    import torch
    if t.dtype == torch.float16:
        return 0
    if t.dtype == torch.bfloat16:
        return 1
    return 2


def flash_block(q, k, v, o, lse=None, causal=False, scale=None) -> FlashBlock:
    """Parameter block for tensors q [B, Sq, H, D], k/v [B, Sk, Hk, D],
    o like q, lse fp32 [B, H, Sq] (or None)."""
    B, Sq, H, D = q.shape
    Sk, Hk = k.shape[1], k.shape[2]
    blk = FlashBlock()
    p = blk.p
    p.q_ptr, p.k_ptr, p.v_ptr, p.o_ptr = (q.data_ptr(), k.data_ptr(), v.data_ptr(),
                                          o.data_ptr())
    p.q_batch_stride, p.q_row_stride, p.q_head_stride = q.stride(0), q.stride(1), q.stride(2)
    p.k_batch_stride, p.k_row_stride, p.k_head_stride = k.stride(0), k.stride(1), k.stride(2)
    p.v_batch_stride, p.v_row_stride, p.v_head_stride = v.stride(0), v.stride(1), v.stride(2)
    p.o_batch_stride, p.o_row_stride, p.o_head_stride = o.stride(0), o.stride(1), o.stride(2)
    p.h, p.h_k, p.h_h_k_ratio = H, Hk, H // Hk
    p.softmax_lse_ptr = lse.data_ptr() if lse is not None else None
    p.b, p.seqlen_q, p.seqlen_k, p.d = B, Sq, Sk, D
    p.seqlen_q_rounded = (Sq + 127) // 128 * 128
    p.seqlen_k_rounded = (Sk + 127) // 128 * 128
    p.d_rounded = D
    p.total_q = B * Sq
    s = (1.0 / math.sqrt(D)) if scale is None else scale
    p.scale_softmax = s
    p.scale_softmax_log2 = s * math.log2(math.e)
    p.p_dropout = 1.0
    p.p_dropout_in_uint8_t = 255
    p.rp_dropout = 1.0
    p.scale_softmax_rp_dropout = s
    p.window_size_left = -1
    p.window_size_right = 0 if causal else -1
    blk.is_bf16 = 1 if _elem(q) == 1 else 0
    blk.is_causal = 1 if causal else 0
    return blk


def flash_forward(q, k, v, o, lse=None, causal=False, scale=None, stream=None) -> int:
    """Calls zlift_flash_fwd; returns 0 done, 1 declined, 2 launch failure."""
    blk = flash_block(q, k, v, o, lse, causal, scale)
    s = 0 if stream is None else int(getattr(stream, "cuda_stream", stream))
    return load().zlift_flash_fwd(ctypes.byref(blk), ctypes.sizeof(blk), _elem(q), s)


def fmha_block(q, k, v, o, lse=None, mask_type=0, scale=None, bias=None) -> FmhaParams:
    """xformers block for q [B, M, H, K], k/v [B, N, H, K], o [B, M, H, K]
    contiguous (o row stride H*K); `bias` [B, H, M, N] of q's type (any
    strides, keys contiguous) is added to the scaled scores."""
    B, M, H, D = q.shape
    N = k.shape[1]
    p = FmhaParams()
    p.query_ptr, p.key_ptr, p.value_ptr = q.data_ptr(), k.data_ptr(), v.data_ptr()
    p.output_ptr = o.data_ptr()
    p.logsumexp_ptr = lse.data_ptr() if lse is not None else None
    p.scale = (1.0 / math.sqrt(D)) if scale is None else scale
    p.head_dim = p.head_dim_value = D
    p.num_queries, p.num_keys, p.num_keys_absolute = M, N, N
    p.custom_mask_type = mask_type
    p.q_strideM, p.k_strideM, p.v_strideM = q.stride(1), k.stride(1), v.stride(1)
    p.o_strideM = o.stride(1)
    p.q_strideH, p.k_strideH, p.v_strideH = q.stride(2), k.stride(2), v.stride(2)
    p.q_strideB, p.k_strideB, p.v_strideB = q.stride(0), k.stride(0), v.stride(0)
    p.num_batches, p.num_heads = B, H
    if bias is not None:
        p.attn_bias_ptr = bias.data_ptr()
        p.bias_strideB, p.bias_strideH, p.bias_strideM = (bias.stride(0), bias.stride(1),
                                                          bias.stride(2))
    return p


def fmha_forward(q, k, v, o, lse=None, mask_type=0, scale=None, stream=None, bias=None) -> int:
    p = fmha_block(q, k, v, o, lse, mask_type, scale, bias)
    s = 0 if stream is None else int(getattr(stream, "cuda_stream", stream))
    return load().zlift_fmha_fwd(ctypes.byref(p), ctypes.sizeof(p), _elem(q), s)
