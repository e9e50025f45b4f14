"""Runtime operations on torch CUDA tensors, each one call into the C ABI (include/mkb_image.h, part 1)."""

import ctypes

from ._lib import lib, check, stream_ptr

ACT_NONE, ACT_GELU_TANH, ACT_SILU, ACT_QUICK_GELU, ACT_GELU_ERF = 0, 1, 2, 3, 4


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
    """Flash attention over head-major q [B][H][Lq_rows][d], k/v [B][H][Lk_rows][d] (d 64 or 128); rows routed into out0
    (joint positions < split) and out1 (see mkb_attention)."""
    B, H, Lq_rows, hd = q.shape
    Lk_rows = k.shape[2]
    Lq = Lq or Lq_rows
    Lk = Lk or Lk_rows
    rows0 = out0.shape[0] // B if out0 is not None else 0
    rows1 = out1.shape[0] // B
    check(lib.mkb_attention(_p(q), Lq, Lq_rows, _p(k), _p(v), Lk, Lk_rows, B, H, hd, q_pos0, mask, cond_len, split,
                            _p(out0), out0.stride(0) if out0 is not None else 0, rows0, _p(out1), out1.stride(0),
                            rows1, stream_ptr()))


def attention_kv_shards(q, k, v, out0, out1, split, Lk, kv_shard_rows, kv_plane_stride, Lq=None, q_pos0=0,
                        mask=MASK_NONE, cond_len=0):
    """attention() with keys and values in shards of kv_shard_rows rows: k and v are [planes][kv_shard_rows][d] and
    key row j of head bh is row j % kv_shard_rows of plane (j // kv_shard_rows) * kv_plane_stride + bh (see
    mkb_attention_kv_shards)."""
    B, H, Lq_rows, hd = q.shape
    Lq = Lq or Lq_rows
    rows0 = out0.shape[0] // B if out0 is not None else 0
    rows1 = out1.shape[0] // B
    check(lib.mkb_attention_kv_shards(_p(q), Lq, Lq_rows, _p(k), _p(v), Lk, Lk, B, H, hd, q_pos0, mask, cond_len,
                                      split, _p(out0), out0.stride(0) if out0 is not None else 0, rows0, _p(out1),
                                      out1.stride(0), rows1, kv_shard_rows, kv_plane_stride, stream_ptr()))


def attention_kv_arriving(q, k, v, out0, out1, split, Lk, kv_shard_rows, kv_plane_stride, own_shard, shard_ready,
                          shard_expect, Lq=None, q_pos0=0):
    """attention_kv_shards() where shard own_shard is complete and every other shard g is read only once the int64
    device flag shard_ready[g] >= shard_expect[0] (see mkb_attention_kv_arriving)."""
    B, H, Lq_rows, hd = q.shape
    Lq = Lq or Lq_rows
    rows0 = out0.shape[0] // B if out0 is not None else 0
    rows1 = out1.shape[0] // B
    check(lib.mkb_attention_kv_arriving(_p(q), Lq, Lq_rows, _p(k), _p(v), Lk, Lk, B, H, hd, q_pos0, MASK_NONE, 0,
                                        split, _p(out0), out0.stride(0) if out0 is not None else 0, rows0, _p(out1),
                                        out1.stride(0), rows1, kv_shard_rows, kv_plane_stride, own_shard,
                                        _p(shard_ready), _p(shard_expect), stream_ptr()))


def attention_wide(qkv, d, n=None, q_col=0, k_col=None, v_col=None, out=None):
    """Single-head attention at head dim 256 / 512 over rows of qkv [n][ld] holding q, k, v side by side (see
    mkb_attention_wide); returns out [n][d] bf16."""
    import torch

    n = n or qkv.shape[0]
    k_col = d if k_col is None else k_col
    v_col = 2 * d if v_col is None else v_col
    if out is None:
        out = torch.empty(n, d, device=qkv.device, dtype=torch.bfloat16)
    check(lib.mkb_attention_wide(_p(qkv), qkv.stride(0), n, d, q_col, k_col, v_col, _p(out), out.stride(0),
                                 stream_ptr()))
    return out


def proj_add(x, w, bias=None, addvec=None, rows_per_sample=None, resid=None, out=None, out_f32=True):
    """y = x @ w.T + bias + addvec[row // rows_per_sample] + resid (fp32 or bf16 out; resid may be out)."""
    import torch

    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty(M, N, device=x.device, dtype=torch.float32 if out_f32 else torch.bfloat16)
    check(lib.mkb_proj_add(_p(x), x.stride(0), _p(w), w.stride(0), _p(bias), _p(addvec),
                           addvec.stride(0) if addvec is not None and addvec.dim() > 1 else 0, rows_per_sample or M,
                           _p(resid), resid.stride(0) if resid is not None else 0, _p(out), out.stride(0),
                           int(out_f32), M, N, K, stream_ptr()))
    return out


def proj_heads(x, w, bias, qh, kh, vh, part0, D, rows_per_sample, pos_offset):
    """Scatter x @ w.T + bias into head-major q/k/v [samples][heads][L][head_dim] (no norm)."""
    M, K = x.shape
    N = w.shape[0]
    ref = next(t for t in (qh, kh, vh) if t is not None)
    L, hd = ref.shape[2], ref.shape[3]
    check(lib.mkb_proj_heads(_p(x), x.stride(0), _p(w), w.stride(0), _p(bias), _p(qh), _p(kh), _p(vh), part0, D, hd,
                             L, rows_per_sample, pos_offset, M, N, K, stream_ptr()))


def proj_geglu(x, w_interleaved, bias=None, out=None):
    import torch

    M, K = x.shape
    N = w_interleaved.shape[0]
    if out is None:
        out = torch.empty(M, N // 2, device=x.device, dtype=torch.bfloat16)
    check(lib.mkb_proj_geglu(_p(x), x.stride(0), _p(w_interleaved), w_interleaved.stride(0), _p(bias), _p(out),
                             out.stride(0), M, N, K, stream_ptr()))
    return out


def conv2d(x, w, taps=9, stride=1, bias=None, addvec=None, resid=None, out=None, out_f32=True):
    """x: channels-last bf16 [B][H][W][C]; w: bf16 [Cout][taps * C]; returns [B][Ho][Wo][Cout]."""
    import torch

    B, H, W, C = x.shape
    Cout = w.shape[0]
    Ho = (H - 1) // stride + 1 if taps == 9 else H
    Wo = (W - 1) // stride + 1 if taps == 9 else W
    if out is None:
        out = torch.empty(B, Ho, Wo, Cout, device=x.device, dtype=torch.float32 if out_f32 else torch.bfloat16)
    check(lib.mkb_conv2d(_p(x), B, H, W, C, _p(w), Cout, taps, stride, _p(bias), _p(addvec),
                         addvec.stride(0) if addvec is not None else 0, _p(resid), Cout if resid is not None else 0,
                         _p(out), Cout, int(out_f32), stream_ptr()))
    return out


def ln_modulate(x, mod, shift=None, eps=1e-6, split=0, mod_stride=0, mod_off=0, out=None):
    """bf16 LayerNorm(x) * (1 + scale) (+ shift) of fp32 rows x [rows][n]; row r's scale is
    mod.flatten()[(r < split ? mod_stride : 0) + mod_off + i] (see mkb_ln_modulate)."""
    import torch

    rows, n = x.shape
    if out is None:
        out = torch.empty(rows, n, device=x.device, dtype=torch.bfloat16)
    check(lib.mkb_ln_modulate(_p(x), _p(mod), _p(shift), _p(out), rows, n, eps, split, mod_stride, mod_off,
                              stream_ptr()))
    return out


def group_norm(x, gamma, beta, groups=32, eps=1e-5, silu=False, out=None):
    """x: fp32 channels-last [B][HW][C] (any shape with that memory order); returns bf16 of the same shape."""
    import torch

    B, C = x.shape[0], x.shape[-1]
    HW = x.numel() // (B * C)
    ws_bytes = lib.mkb_group_norm_workspace_size(B, HW, C, groups)
    ws = torch.empty(max(ws_bytes, 16) // 4 + 1, device=x.device, dtype=torch.float32)
    if out is None:
        out = torch.empty(x.shape, device=x.device, dtype=torch.bfloat16)
    check(lib.mkb_group_norm(_p(x), _p(out), _p(gamma), _p(beta), B, HW, C, groups, eps, int(silu), _p(ws),
                             ws.numel() * 4, stream_ptr()))
    return out
