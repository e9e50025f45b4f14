/* mkb_image.h: the C ABI of the B200 denoiser hot path.
 *
 * Two layers, both plain C (pointers, sizes, status codes; no C++ or torch types):
 *
 *  1. Runtime operations on caller-owned DEVICE memory. They replace the GPU runtime calls the reference's model
 *     code makes per step (mako-common's TransformerRuntime: proj / attention / heads_norm / norm, and the
 *     src/kernels/image.metal kernels ln_modulate and gate_add). Each takes a CUDA stream (NULL: the legacy stream)
 *     and only enqueues work.
 *
 *  2. A denoiser handle (mkb_dit) that owns its weights and device buffers and exposes the reference's model
 *     interface, image::Engine::begin / step (src/image/engine.hpp:165-166), on HOST buffers.
 *
 * Errors: every entry point returns MKB_OK or an error code; mkb_last_error() gives a message for the calling
 * thread. No C++ exception crosses this boundary.
 */
#ifndef MKB_IMAGE_H
#define MKB_IMAGE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum mkb_status {
    MKB_OK = 0,
    MKB_ERR_INVALID = 1, /* bad argument (null pointer, unsupported size, misaligned pointer) */
    MKB_ERR_CUDA = 2,    /* a CUDA runtime call failed */
    MKB_ERR_STATE = 3,   /* call out of order (step before begin, unknown slot) */
    MKB_ERR_KERNEL = 4,  /* a kernel reported an error (a bounded wait timed out); see mkb_last_error() */
    MKB_ERR_ALLOC = 5    /* device memory allocation failed */
} mkb_status;

/* The message of the last error on this thread ("" if none). */
const char* mkb_last_error(void);

/* Activations a projection epilogue can apply. */
enum { MKB_ACT_NONE = 0, MKB_ACT_GELU_TANH = 1, MKB_ACT_SILU = 2 };

/* ---------------------------------------------------------------------------------------------------------------
 * Runtime operations (device pointers). bf16 matrices are row-major with the given leading dimension in elements.
 * ------------------------------------------------------------------------------------------------------------- */

/* y[M][N] = act(x[M][K] * w[N][K]^T + bias[N]). y is bf16 (out_f32 = 0) or fp32 (out_f32 = 1).
 * Replaces TransformerRuntime::proj() (called e.g. at src/image/qwen_image.cpp:196-215,224,272,277,281,288) and the
 * activation kernels that follow it (gelu_tanh at qwen_image.cpp:211, silu at :198,202). */
mkb_status mkb_proj(const void* x, long ldx, const void* w, long ldw, const float* bias, void* y, long ldy, int M,
                    int N, int K, int act, int out_f32, void* stream);

/* resid[M][N] += g * (x * w^T + bias), g = gate[row / rows_per_sample][col] (tanh(gate) when tanh_gate != 0, the
 * reference's gate_add, src/kernels/image.metal:56-65). resid is fp32 with leading dimension ldr; the gate rows of
 * consecutive samples are gate_stride floats apart. Replaces proj() + gate_add (qwen_image.cpp:272-274, 281-282). */
mkb_status mkb_proj_gate_add(const void* x, long ldx, const void* w, long ldw, const float* bias, float* resid,
                             long ldr, const float* gate, long gate_stride, int rows_per_sample, int tanh_gate, int M,
                             int N, int K, void* stream);

/* The fused QKV projection: [q | k | v] = x * w^T + bias with N = 3 * heads * 128. q and k are RMS-normed per
 * 128-wide head (weights norm_q / norm_k, eps) and rotated by the RoPE table rope[L][64][2] (cos, sin of each
 * interleaved pair; NULL: no rotation), then written as bf16 into q/k/v heads [samples][heads][L][128]: row r of x
 * goes to sample r / rows_per_sample, position pos_offset + r % rows_per_sample. Replaces proj() +
 * heads_norm_half x2 + heads_half (qwen_image.cpp:224-250). */
mkb_status mkb_proj_qkv_heads(const void* x, long ldx, const void* w, long ldw, const float* bias,
                              const float* norm_q, const float* norm_k, const float* rope, void* qh, void* kh,
                              void* vh, int heads, int L, int rows_per_sample, int pos_offset, float eps, int M, int K,
                              void* stream);

/* SwiGLU projection: w holds (gate | up) rows interleaved in blocks (see mkb_swiglu_interleave); the
 * output is y[M][N/2] = silu(gate) * up, bf16. Replaces proj(gate_up) + swiglu_rows (qwen_image.cpp:277-280). */
mkb_status mkb_proj_swiglu(const void* x, long ldx, const void* w, long ldw, const float* bias, void* y, long ldy,
                           int M, int N, int K, void* stream);

/* Block size of the gate/up row interleave mkb_proj_swiglu expects: rows [2*j*B, 2*j*B + B) of the interleaved
 * matrix are gate rows [j*B, (j+1)*B), the next B rows the matching up rows. */
int mkb_swiglu_interleave(void);

/* Attention masks. */
enum { MKB_MASK_NONE = 0, MKB_MASK_COND_CAUSAL = 1 };

/* Flash attention, head dim 128: out = softmax(q k^T / sqrt(128)) v per (sample, head). q is [B][H][Lq_rows][128],
 * k and v [B][H][Lk_rows][128] (bf16, head-major, as mkb_proj_qkv_heads writes them); the first Lq query rows and Lk
 * keys are used. Query row i sits at joint position q_pos0 + i; keys at positions 0..Lk-1. MKB_MASK_COND_CAUSAL: a
 * query at position < cond_len sees keys < cond_len only (the reference's text rows, which is what lets it cache the
 * text K/V; qwen_image.cpp:251-271). Output rows are bf16 [.][H*128]: position p < split goes to row
 * (b * rows0 + p) of out0, otherwise row (b * rows1 + p - split) of out1 (the text and image streams' inputs of the
 * output projection). Replaces TransformerRuntime::attention() (qwen_image.cpp:271). */
mkb_status mkb_attention(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk, int Lk_rows, int B,
                         int H, int q_pos0, int mask, int cond_len, int split, void* out0, long ld0, int rows0,
                         void* out1, long ld1, int rows1, void* stream);

/* The status word kernels write their error bits to (device memory owned by the library; 0 = no error). Reads and
 * clears it: returns MKB_OK, or MKB_ERR_KERNEL with the bits in *bits. Synchronises the device. */
mkb_status mkb_check_kernels(uint32_t* bits);

#ifdef __cplusplus
}
#endif

#endif /* MKB_IMAGE_H */
