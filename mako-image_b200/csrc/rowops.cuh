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
    int affine = 0;  // 1: y = norm * scale + shift (a plain LayerNorm with weight and bias)
};
cudaError_t ln_modulate(const LnModArgs& a, cudaStream_t st);
// Both row sets (same D) in one launch.
cudaError_t ln_modulate2(const LnModArgs& a, const LnModArgs& b, cudaStream_t st);

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
// apart), fp32 out (rows ldy apart). act: 0 none, 2 silu (GemmArgs's Act values). no_smem: x read through L1 (x and
// ldx 16-byte aligned) instead of staged in shared memory, so that the blocks can share SMs with a GEMM's; the same
// results.
cudaError_t gemv(const __nv_bfloat16* W, const float* x, long ldx, const float* bias, float* y, long ldy, int B,
                 int N, int K, int act, cudaStream_t st, bool no_smem = false);

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

// GroupNorm over channels-last fp32 x [B][HW][C] (groups of C / groups consecutive channels, statistics over the
// group's channels of all HW pixels of a sample), then y = norm * gamma + beta, optionally SiLU, as bf16. The
// runtime's group_norm (called at sdxl.cpp:728,732,762,941 and engine.cpp:726). Two passes: per-chunk (count, mean,
// M2) partials combined with Chan's parallel update, then the apply pass. `ws` is scratch of
// group_norm_workspace() bytes.
struct GnArgs {
    const float* x;
    __nv_bfloat16* y;
    const float* gamma;
    const float* beta;
    int B, HW, C, groups;
    float eps;
    int silu;
    float* ws;
};
size_t group_norm_workspace(int B, int HW, int C, int groups);
cudaError_t group_norm(const GnArgs& a, cudaStream_t st);
// The same with the statistics pass already done by the convolution that wrote x (GemmArgs::gn_part): parts holds
// float4 (count, mean, M2, 0) per [B][groups][nchunks]; a.ws (16-byte aligned) needs B * groups * 128 floats.
cudaError_t group_norm_from_parts(const GnArgs& a, const float4* parts, int nchunks, cudaStream_t st);

// Nearest 2x upsampling of channels-last fp32 x [B][H][W][C] into bf16 y [B][2H][2W][C] (the upsample2x kernel,
// src/kernels/image.metal:77-84), ready as a convolution input.
cudaError_t upsample2x_bf16(const float* x, __nv_bfloat16* y, int B, int H, int W, int C, cudaStream_t st);

// y[p] = [a[p] | b[p]] for pixels p: channel concatenation of fp32 [P][Ca] and [P][Cb] (the skip concat of the
// UNet's up blocks, sdxl.cpp:910-918).
cudaError_t concat_channels(const float* a, int Ca, const float* b, int Cb, float* y, long P, cudaStream_t st);

// y[p][0:C] = bf16(x[p][0:C]), y[p][C:Cp] = 0: a thin input (latents) widened to a multiple of 64 channels for the
// convolution.
cudaError_t pad_channels_bf16(const float* x, int C, __nv_bfloat16* y, int Cp, long P, cudaStream_t st);

// Latent tokens [B][gh*gw][16] (channel, row, column of a 2x2 patch) to the channels-last image bf16
// [B][2gh][2gw][Cp] times `scale`, channels 4..Cp-1 zero (sdxl.cpp:80-87, engine.cpp:888-898).
cudaError_t unpack_tokens_bf16(const float* tokens, __nv_bfloat16* img, int B, int gh, int gw, int Cp, float scale,
                               cudaStream_t st);
// The inverse for the first 4 of Cs channels of fp32 img [B][2gh][2gw][Cs] (sdxl.cpp:946-952).
cudaError_t pack_tokens(const float* img, int Cs, float* tokens, int B, int gh, int gw, cudaStream_t st);
// One image's tokens [gh*gw][4 z] (z latent channels in 2x2 patches) to its channels-last latent image
// [2gh][2gw][Cp] bf16, value i of a token mapped to v * affine[i] + affine[4 z + i].
cudaError_t unpack_tokens_affine_bf16(const float* tokens, __nv_bfloat16* img, int gh, int gw, int z, int Cp,
                                      const float* affine, cudaStream_t st);
// out[i] = silu(a[i] + b[i]).
cudaError_t add_silu(const float* a, const float* b, float* out, uint64_t n, cudaStream_t st);
// RGBA [B][H][W][4] = clamp(img[..][0:3], -1, 1), alpha 1, from fp32 img with Cs channels per pixel
// (engine.cpp:948-953).
cudaError_t to_rgba(const float* img, int Cs, float* rgba, long P, cudaStream_t st);
// Row softmax of scale * s (fp32 [rows][n]) into bf16 p (softmax_rows, src/kernels/image.metal:101-128).
cudaError_t softmax_rows_bf16(const float* s, __nv_bfloat16* p, long rows, int n, float scale, cudaStream_t st);
// y[c][r] = x[r][c0 + c] for rows r < rows, c < cols of bf16 x with row stride ldx (transpose_f32 / copy_cols,
// image.metal:134-147): V^T for the VAE's mid attention.
cudaError_t transpose_bf16(const __nv_bfloat16* x, long ldx, int c0, __nv_bfloat16* y, long rows, int cols,
                           cudaStream_t st);

// SDXL's text encoders (Sdxl::encode_clip, sdxl.cpp:459-546).
// x [M][E] fp32 = tok[ids[m]] + pos[m % T]: token plus position embeddings (ids checked by the caller).
cudaError_t clip_embed(const int* ids, const float* tok, const float* pos, float* x, int M, int T, int E,
                       cudaStream_t st);
// LayerNorm (gamma g, beta b) of fp32 rows x [M][E] into y [M][2E] bf16: y[m][e] the bf16 rounding of the normed value
// v, y[m][E + e] the bf16 rounding of v minus it. A GEMM over K = 2E against weights duplicated along K then
// multiplies v to within ~2^-16: the split the reference's text-encoder GEMMs use (docs/architecture.md:9-11).
cudaError_t ln_split_bf16(const float* x, const float* g, const float* b, __nv_bfloat16* y, int M, int E, float eps,
                          cudaStream_t st);
// The same split of fp32 x [M][N] into y [M][2N] bf16.
cudaError_t split_bf16(const float* x, __nv_bfloat16* y, long M, int N, cudaStream_t st);
// out [B][P] = LayerNorm(x row (b * T + eos[b])) times proj [E][P] (bigG's pooled state, sdxl.cpp:521-541); E <= 2048.
cudaError_t clip_pooled(const float* x, const int* eos, const float* g, const float* b, const float* proj, float* out,
                        int B, int T, int E, int P, float eps, cudaStream_t st);

// x[i] += dt * (v_u[i] + g * (v_c[i] - v_u[i])) (classifier-free guidance then an Euler step, engine.cpp:476-480,
// :500-503); with v_u null: x += dt * v_c.
cudaError_t cfg_euler(float* x, const float* v_c, const float* v_u, float g, float dt, uint64_t n, cudaStream_t st);

}  // namespace mkb
