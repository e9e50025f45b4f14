// Memory-bound row and element kernels of the denoiser step: modulated LayerNorm, RMSNorm, the fp32-activation GEMV
// of the time path, the timestep sinusoid, the seeded normal generator, casts, head-row copies and the fused
// CFG + Euler update. Each is one HBM pass with 128-bit accesses.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace mkb {

// y[row] = LayerNorm(x[row]) * (1 + scale) + shift (no affine; eps), bf16 out. The modulation of row r is that of
// sample s = r / rows_per_sample at scale + s * mod_stride (shift likewise; shift may be null). Rows whose index
// within the sample is < split take scale + alt_off instead (the reference's text rows use modulation row 1,
// src/kernels/image.metal:33-53).
struct LnModArgs {
    const float* x;
    __nv_bfloat16* y;
    const float* scale;
    const float* shift;
    long mod_stride;
    long alt_off;
    int split;
    int rows, D, rows_per_sample;
    float eps;
};
cudaError_t ln_modulate(const LnModArgs& a, cudaStream_t st);

// y[row] = x[row] / rms(x[row]) * w, fp32 in, bf16 out. Sample s's rows come from src[s] (rows_per_sample each).
struct RmsArgs {
    const float* src[8];
    __nv_bfloat16* y;
    const float* w;
    int samples, rows_per_sample, C;
    float eps;
};
cudaError_t rms_norm_rows(const RmsArgs& a, cudaStream_t st);

// y[b][n] = act(W[n] . x[b] + bias[n]) for b < B (B <= 8): bf16 weights [N][K], fp32 activations [B][K] (rows ldx
// apart), fp32 out (rows ldy apart). act: 0 none, 2 silu (GemmArgs's Act values).
cudaError_t gemv(const __nv_bfloat16* W, const float* x, long ldx, const float* bias, float* y, long ldy, int B,
                 int N, int K, int act, cudaStream_t st);

// tp[r][0:128] = cos(1000 t_r f_i), tp[r][128:256] = sin(1000 t_r f_i), f_i = exp(-ln(10000) i / 128), for the rows'
// noise levels t (qwen_image.cpp:179-187).
cudaError_t timestep_sinusoid(const float* t, float* tp, int rows, cudaStream_t st);

// out[i] = mean + std * N(0, 1) of the counter-based stream `key` at element offset + i (the generator of the
// oracle's rng.normal); bf16 or fp32 output.
cudaError_t fill_normal(void* out, bool bf16, uint64_t n, uint64_t key, uint64_t offset, float std, float mean,
                        cudaStream_t st);

cudaError_t cast_f32_bf16(const float* x, __nv_bfloat16* y, uint64_t n, cudaStream_t st);

// y[i] = silu(x[i]) (fp32).
cudaError_t silu_f32(const float* x, float* y, uint64_t n, cudaStream_t st);

// Copies `rows` rows of 128 bf16 for each of `heads` (sample, head) pairs: dst[h][dst_off + r] = src[h][src_off + r],
// with src_rows / dst_rows rows per head (the text K/V cache in and out of the attention layout).
cudaError_t copy_head_rows(const __nv_bfloat16* src, int src_rows, int src_off, __nv_bfloat16* dst, int dst_rows,
                           int dst_off, int heads, int rows, cudaStream_t st);

// x[i] += dt * (v_u[i] + g * (v_c[i] - v_u[i])) (classifier-free guidance then an Euler step, engine.cpp:476-480,
// :500-503); with v_u null: x += dt * v_c.
cudaError_t cfg_euler(float* x, const float* v_c, const float* v_u, float g, float dt, uint64_t n, cudaStream_t st);

}  // namespace mkb
