"""Runtime operations on torch CUDA tensors, each one call into the C ABI (include/mkb_image.h, part 1)."""

import ctypes

from ._lib import lib, check, stream_ptr

ACT_NONE, ACT_GELU_TANH, ACT_SILU = 0, 1, 2


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def proj(x, w, bias=None, act=ACT_NONE, out=None, out_f32=False):
    """y = act(x @ w.T + bias); x [M][K] bf16, w [N][K] bf16, bias fp32 [N]."""
    import torch

    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=torch.float32 if out_f32 else torch.bfloat16)
    check(lib.mkb_proj(_p(x), x.stride(0), _p(w), w.stride(0), _p(bias), _p(out), out.stride(0), M, N, K, act,
                       int(out_f32), stream_ptr()))
    return out


def proj_gate_add(x, w, resid, gate, bias=None, rows_per_sample=None, tanh_gate=False):
    """resid += g(gate[row // rows_per_sample]) * (x @ w.T + bias), in place; gate [samples][N] fp32."""
    M, K = x.shape
    N = w.shape[0]
    rps = rows_per_sample or M
    check(lib.mkb_proj_gate_add(_p(x), x.stride(0), _p(w), w.stride(0), _p(bias), _p(resid), resid.stride(0),
                                _p(gate), gate.stride(0) if gate.dim() > 1 else 0, rps, int(tanh_gate), M, N, K,
                                stream_ptr()))
    return resid


def proj_qkv_heads(x, w, bias, norm_q, norm_k, rope, qh, kh, vh, rows_per_sample, pos_offset, eps=1e-6):
    """Fused QKV projection into head-major q/k/v [samples][heads][L][128] (bf16)."""
    M, K = x.shape
    heads, L = qh.shape[1], qh.shape[2]
    check(lib.mkb_proj_qkv_heads(_p(x), x.stride(0), _p(w), w.stride(0), _p(bias), _p(norm_q), _p(norm_k), _p(rope),
                                 _p(qh), _p(kh), _p(vh), heads, L, rows_per_sample, pos_offset, eps, M, K,
                                 stream_ptr()))


def proj_swiglu(x, w_interleaved, bias=None, out=None):
    """silu(gate) * up from a gate/up-interleaved weight (see swiglu_interleave)."""
    import torch

    M, K = x.shape
    N = w_interleaved.shape[0]
    if out is None:
        out = torch.empty(M, N // 2, device=x.device, dtype=torch.bfloat16)
    check(lib.mkb_proj_swiglu(_p(x), x.stride(0), _p(w_interleaved), w_interleaved.stride(0), _p(bias), _p(out),
                              out.stride(0), M, N, K, stream_ptr()))
    return out


def swiglu_interleave_block():
    return lib.mkb_swiglu_interleave()


def check_kernels():
    bits = ctypes.c_uint32(0)
    check(lib.mkb_check_kernels(ctypes.byref(bits)))
    return bits.value


MASK_NONE, MASK_COND_CAUSAL = 0, 1


def attention(q, k, v, out0, out1, split, Lq=None, Lk=None, q_pos0=0, mask=MASK_NONE, cond_len=0):
    """Flash attention over head-major q [B][H][Lq_rows][128], k/v [B][H][Lk_rows][128]; rows routed into out0
    (joint positions < split) and out1 (see mkb_attention)."""
    B, H, Lq_rows, _ = q.shape
    Lk_rows = k.shape[2]
    Lq = Lq or Lq_rows
    Lk = Lk or Lk_rows
    rows0 = out0.shape[0] // B if out0 is not None else 0
    rows1 = out1.shape[0] // B
    check(lib.mkb_attention(_p(q), Lq, Lq_rows, _p(k), _p(v), Lk, Lk_rows, B, H, q_pos0, mask, cond_len, split,
                            _p(out0), out0.stride(0) if out0 is not None else 0, rows0, _p(out1), out1.stride(0),
                            rows1, stream_ptr()))
