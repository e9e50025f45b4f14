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

/* Kernel launches this library has made in this process (all threads, all devices). */
uint64_t mkb_kernel_launches(void);

/* Activations a projection epilogue can apply (quick GELU x sigmoid(1.702 x) and the erf GELU: the CLIP text
 * encoders' fc1, src/image/sdxl.cpp:508). */
enum { MKB_ACT_NONE = 0, MKB_ACT_GELU_TANH = 1, MKB_ACT_SILU = 2, MKB_ACT_QUICK_GELU = 3, MKB_ACT_GELU_ERF = 4 };

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

/* y = x * w^T + bias + addvec[row / rows_per_sample] + resid (each optional: NULL), y fp32 (out_f32 = 1) or bf16.
 * resid is fp32 [M][N] rows ld_resid apart and may be y itself (an in-place residual add). The projections of the
 * SDXL UNet's transformer blocks with their residual adds (sdxl.cpp:763-795). */
mkb_status mkb_proj_add(const void* x, long ldx, const void* w, long ldw, const float* bias, const float* addvec,
                        long addvec_stride, int rows_per_sample, const float* resid, long ld_resid, void* y, long ldy,
                        int out_f32, int M, int N, int K, void* stream);

/* y = x * w^T + bias scattered into head-major bf16 [samples][heads][L][head_dim]: columns [p*D, (p+1)*D) go to part
 * part0 + p of (q, k, v), head h at columns h*head_dim of its part; row r to sample r / rows_per_sample, position
 * pos_offset + r % rows_per_sample of L. No norm (SDXL's q, k, v and the cached cross-attention k, v, sdxl.cpp:
 * 443-457, 701-717). */
mkb_status mkb_proj_heads(const void* x, long ldx, const void* w, long ldw, const float* bias, void* qh, void* kh,
                          void* vh, int part0, int D, int head_dim, int L, int rows_per_sample, int pos_offset, int M,
                          int N, int K, void* stream);

/* GEGLU projection: w holds (hidden | gate) rows interleaved in blocks of mkb_swiglu_interleave(); the output is
 * y[M][N/2] = hidden * GELU_erf(gate), bf16 (geglu_rows, src/kernels/image.metal:476-484). */
mkb_status mkb_proj_geglu(const void* x, long ldx, const void* w, long ldw, const float* bias, void* y, long ldy,
                          int M, int N, int K, void* stream);

/* Convolution on channels-last bf16 input x [B][H][W][C] (C a multiple of 64) with weights w [Cout][taps][C] bf16
 * (taps 9: 3x3 with padding 1, stride 1 or 2; taps 1: 1x1), as an implicit GEMM on the tensor cores (no im2col
 * buffer: each 3x3 tap is a shifted window of the input, zero outside the image). Epilogue as mkb_proj_add with
 * rows = output pixels (b * Ho + y) * Wo + x and addvec per image. Replaces ConvRuntime::conv (sdxl.cpp:729-735,
 * engine.cpp:737-741, 904-943). The output width must be a multiple of 8. */
mkb_status mkb_conv2d(const void* x, int B, int H, int W, int C, const void* w, int Cout, int taps, int stride,
                      const float* bias, const float* addvec, long addvec_stride, const float* resid, long ld_resid,
                      void* y, long ldy, int out_f32, void* stream);

/* LayerNorm without weights, times (1 + scale), plus an optional shift, of `rows` rows of n floats; y is bf16 (the
 * next projection's input). Row r's scale is mod[(r < split ? mod_stride : 0) + mod_off + i] and its shift, when
 * shift is not null, shift at the same offset: the reference's ln_modulate (src/kernels/image.metal:33-53, ModArgs
 * :23-30, dispatched by qwen_image.cpp:223, 276, 286), whose shift-less form is shift == NULL. n a multiple of 128,
 * at most 4096; x, mod + mod_off and shift + mod_off 16-byte aligned, mod_stride a multiple of 4. */
mkb_status mkb_ln_modulate(const float* x, const float* mod, const float* shift, void* y, long rows, int n, float eps,
                           long split, long mod_stride, long mod_off, void* stream);

/* GroupNorm of channels-last fp32 x [B][HW][C] (C / groups consecutive channels per group), y = norm * gamma + beta,
 * then SiLU if silu != 0, bf16 out. workspace: device scratch of mkb_group_norm_workspace_size() bytes. The
 * runtime's group_norm (sdxl.cpp:728-762, engine.cpp:722-730). */
size_t mkb_group_norm_workspace_size(int B, int HW, int C, int groups);
mkb_status mkb_group_norm(const float* x, void* y, const float* gamma, const float* beta, int B, int HW, int C,
                          int groups, float eps, int silu, void* workspace, size_t workspace_bytes, void* stream);

/* GroupNorm exactly as mkb_group_norm, but with no workspace argument and no allocation: the statistics scratch is
 * a fixed array built into the library (mkb_group_norm_static_max_bytes(), 4 MiB, held on every device that loads
 * the library until the process exits). For callers that cannot allocate device memory or hand over a scratch
 * buffer: code running while another component owns all device memory (a serving loop behind a caching allocator),
 * real-time paths that must not risk an allocation's latency or failure, and hosts that only pass in tensors they
 * already own. No counterpart in the reference (its runtime owns its scratch buffers).
 * Limits: sizes whose statistics need more than the built-in scratch (mkb_group_norm_workspace_size() above
 * mkb_group_norm_static_max_bytes()) are rejected with MKB_ERR_INVALID. That size is B * nchunks * groups * 12 +
 * B * groups * 8 bytes, with B * nchunks about 1184 (eight statistics chunks per SM) for large images and
 * B * ceil(HW / 16) for small ones: about groups * 14 KB, so up to roughly 290 groups fit whatever the image size. The first call on a device looks up the scratch's device address (once per device, with that
 * device current); make that first call before any stream capture. That address is kept for the life of the
 * process, so do not call this entry point on a device after cudaDeviceReset of it. All calls on a device share the one scratch
 * array and it keeps the last call's contents (nothing in it needs clearing: each call writes every entry it reads
 * first), so calls that overlap on the GPU (different streams, or threads) race; serialise them. */
size_t mkb_group_norm_static_max_bytes(void);
mkb_status mkb_group_norm_static(const float* x, void* y, const float* gamma, const float* beta, int B, int HW, int C,
                                 int groups, float eps, int silu, void* stream);

/* Attention masks. */
enum { MKB_MASK_NONE = 0, MKB_MASK_COND_CAUSAL = 1 };

/* Flash attention, head dim d = 64 or 128: out = softmax(q k^T / sqrt(d)) v per (sample, head). q is
 * [B][H][Lq_rows][d], k and v [B][H][Lk_rows][d] (bf16, head-major, as mkb_proj_qkv_heads / mkb_proj_heads write
 * them); the first Lq query rows and Lk keys are used. Query row i sits at joint position q_pos0 + i; keys at
 * positions 0..Lk-1. MKB_MASK_COND_CAUSAL (the runtime's `block` argument, qwen_image.cpp:271 and sdxl.cpp:501): a
 * query at position p < cond_len sees keys 0..p only, causal and never a later row (the reference's text rows, which
 * is what lets it cache the text K/V, qwen_image.cpp:251-262); queries at p >= cond_len see every key. cond_len >= Lk
 * is plain causal attention (the CLIP encoders' block = UINT32_MAX). Output rows are bf16 [.][H*128]: position p < split goes to row
 * (b * rows0 + p) of out0, otherwise row (b * rows1 + p - split) of out1 (the text and image streams' inputs of the
 * output projection; columns [h * d, h * d + d)). Replaces TransformerRuntime::attention() (qwen_image.cpp:271) and the
 * hd-64 flash_attn_coop_64_32 the SDXL UNet calls (sdxl.cpp:450-457). */
mkb_status mkb_attention(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk, int Lk_rows, int B,
                         int H, int head_dim, int q_pos0, int mask, int cond_len, int split, void* out0, long ld0,
                         int rows0, void* out1, long ld1, int rows1, void* stream);

/* mkb_attention over keys and values split into shards of kv_shard_rows rows (a multiple of 128), the layout a
 * sequence-parallel all-gather leaves: key row j of head (b, h) is row j % kv_shard_rows of head-plane
 * (j / kv_shard_rows) * kv_plane_stride + b * H + h of k (and of v), each plane kv_shard_rows x d. No counterpart in
 * the reference, which runs on one device; mkb_dit's sequence-parallel step uses the same kernel path. */
mkb_status mkb_attention_kv_shards(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk,
                                   int Lk_rows, int B, int H, int head_dim, int q_pos0, int mask, int cond_len,
                                   int split, void* out0, long ld0, int rows0, void* out1, long ld1, int rows1,
                                   int kv_shard_rows, int kv_plane_stride, void* stream);

/* Single-head attention at head dim d = 256 or 512: the VAE decoder's mid-block attention over every pixel of the
 * latent image (Engine::vae_attention, src/image/engine.cpp:748-778, which runs it as a score GEMM, a row softmax and
 * a P V GEMM; here one flash kernel). q, k and v of n rows sit side by side in one bf16 buffer (rows of ld elements,
 * at columns q_col, k_col and v_col, multiples of 64); out (bf16, rows ldo apart) = softmax(q k^T / sqrt(d)) v. */
mkb_status mkb_attention_wide(const void* qkv, long ld, int n, int d, int q_col, int k_col, int v_col, void* out,
                              long ldo, void* stream);

/* The same over shards that other ranks copy into this GPU's memory while the kernel runs (the sequence-parallel
 * peer exchange; no counterpart in the reference, which runs on one device). Shard own_shard is complete at launch;
 * before reading any other shard g the kernel waits until the 64-bit device flag shard_ready[g] >= *shard_expect
 * (both device pointers; an acquire load at system scope). Every CTA starts at its own shard's keys and wraps round,
 * so only the online softmax's rounding differs from mkb_attention_kv_shards. A flag that does not reach the value
 * within 2 s ends the launch; mkb_check_kernels then reports MKB_ERR_KERNEL with bit 0x100. mask must be
 * MKB_MASK_NONE. */
mkb_status mkb_attention_kv_arriving(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk,
                                     int Lk_rows, int B, int H, int head_dim, int q_pos0, int mask, int cond_len,
                                     int split, void* out0, long ld0, int rows0, void* out1, long ld1, int rows1,
                                     int kv_shard_rows, int kv_plane_stride, int own_shard,
                                     const unsigned long long* shard_ready, const unsigned long long* shard_expect,
                                     void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * The denoiser (image::Engine's model interface, src/image/engine.hpp:158-166, on the Qwen-Image-style MMDiT).
 * ------------------------------------------------------------------------------------------------------------- */

/* Variants: MKB_VARIANT_QWEN1 is the Qwen-Image(-1) MMDiT shape (separate text/image weights with biases, per-block
 * AdaLN shift/scale/gate, GELU-tanh FFN, joint attention); MKB_VARIANT_REF21 is the reference's own block math
 * (src/image/qwen_image.cpp:144-293: shared weights, one shared modulation, tanh gates, SwiGLU, condition-causal
 * attention with the text K/V cached after a slot's first step). */
enum { MKB_VARIANT_QWEN1 = 0, MKB_VARIANT_REF21 = 1 };

typedef struct mkb_dit_config {
    int variant;
    int hidden;           /* D = heads * 128 */
    int heads;
    int ffn;              /* F (qwen1: GELU width; ref21: SwiGLU width) */
    int blocks;
    int text_dim;         /* width of the prompt embeddings, a multiple of 128 */
    int max_batch;        /* samples per step call, 1..8 */
    int max_text_tokens;  /* S */
    int max_image_tokens; /* N = h * w */
    int slots;            /* text conditionings kept (the reference's slot argument; 2 = cond / uncond) */
} mkb_dit_config;

typedef struct mkb_dit mkb_dit;

/* Creates a denoiser on the current CUDA device: allocates weights and step buffers for the configured maxima.
 * Weights start at zero; fill them with mkb_dit_init_random or mkb_dit_weight_write. */
mkb_status mkb_dit_create(const mkb_dit_config* cfg, mkb_dit** out);
void mkb_dit_destroy(mkb_dit* d);

/* Synthetic weights from a seed: weight i is filled from the normal stream tensor_key(seed, i) (splitmix64 based,
 * the generator of oracle/rng.py) with std `std` (norm scales: 1 + 0.1 N(0,1)). */
mkb_status mkb_dit_init_random(mkb_dit* d, uint64_t seed, float std);

/* Weight table: count, and name / shape (rows, cols; cols = 0 for vectors) of entry i. Names follow the reference's
 * module names in short form ("blk3.img.qkv.w", "time.lin1.w", ...); matrices are stored bf16, vectors fp32. */
int mkb_dit_weight_count(const mkb_dit* d);
mkb_status mkb_dit_weight_info(const mkb_dit* d, int i, const char** name, long* rows, long* cols);
/* Copies a weight to / from host fp32 (matrices are rounded to bf16 on write). The reference's row order is kept:
 * a SwiGLU gate_up matrix is [gate rows; up rows] here even though the device interleaves it. */
mkb_status mkb_dit_weight_read(mkb_dit* d, const char* name, float* host);
mkb_status mkb_dit_weight_write(mkb_dit* d, const char* name, const float* host);

/* ---- Weights from files (replaces QwenImage::load_transformer, src/image/qwen_image.cpp:79-111, and
 * Engine::add_lora / QwenImage::lora_target, src/image/engine.hpp:195-197, qwen_image.cpp:295-331). */

/* The handle's variant (MKB_VARIANT_*), or -1 for a null handle. */
int mkb_dit_variant(const mkb_dit* d);
/* Rows [row0, row0 + rows) of weight `name` from host fp32 [rows][cols] (a vector's elements for cols 0). */
mkb_status mkb_dit_weight_write_rows(mkb_dit* d, const char* name, long row0, long rows, const float* host);
/* W[row0 .. row0 + rows) += scale * B A on the device, W a matrix of the table, A [rank][cols] and B [rows][rank]
 * host fp32 (rank <= 512). */
mkb_status mkb_dit_weight_lora_rows(mkb_dit* d, const char* name, long row0, long rows, const float* A,
                                    const float* B, int rank, float scale);
/* Loads safetensors checkpoint files (F32 / F16 / BF16) by the checkpoint's tensor names: the reference's for
 * MKB_VARIANT_REF21 (q/k/v and gate/up row-stacked, txt_in.text_norm stored zero-centred), the published Qwen-Image
 * transformer's for MKB_VARIANT_QWEN1 (img_mod.1, attn.to_q / add_q_proj, img_mlp.net.0.proj, ... with biases).
 * Tensors must match the model's shapes. strict != 0: an unknown tensor, or a weight the files leave unwritten, is
 * an error. *loaded (optional) counts the tensors written. */
mkb_status mkb_dit_load_safetensors(mkb_dit* d, const char* const* paths, int n_paths, int strict, int* loaded);
/* Merges one LoRA pair into the module's rows, W += scale * B A: `module` by checkpoint name without ".weight"
 * ("transformer_blocks.3.attn.to_q", "img_mlp.gate_up", ...), A [rank][in_features], B [out_features][rank]. */
mkb_status mkb_dit_lora_merge(mkb_dit* d, const char* module, const float* A, const float* B, int rank,
                              int in_features, int out_features, float scale);
/* Merges every pair of a LoRA safetensors file: <module>.lora_A / lora_B (or lora_down / lora_up) .weight, with an
 * optional scalar <module>.alpha scaling by alpha / rank; "transformer." / "diffusion_model." prefixes are dropped.
 * *merged (optional) counts the modules. */
mkb_status mkb_dit_load_lora(mkb_dit* d, const char* path, float scale, int* merged);

/* The safetensors reader behind the loaders, for callers that inspect files. */
typedef struct mkb_st_file mkb_st_file;
mkb_status mkb_st_open(const char* path, mkb_st_file** out);
void mkb_st_close(mkb_st_file* f);
int mkb_st_count(const mkb_st_file* f);
/* Tensor i: name, dtype as written ("F32", "BF16", ...), up to 8 dims. */
mkb_status mkb_st_info(const mkb_st_file* f, int i, const char** name, const char** dtype, int64_t* dims, int* ndim);
/* Tensor `name` as fp32 (F32 / F16 / BF16 files); count must equal its element count. */
mkb_status mkb_st_read_f32(const mkb_st_file* f, const char* name, float* out, int64_t count);

/* Engine::begin (engine.hpp:165): prompt embeddings [S][text_dim] (host fp32) for `slot` on an h x w token grid.
 * Slots share the grid (the last begin sets it). Resets the slot's step count (ref21: its text K/V cache). */
mkb_status mkb_dit_begin(mkb_dit* d, const float* prompt, int S, int h, int w, int slot);

/* Engine::step (engine.hpp:166): the velocity out[N][64] for latents[N][64] at noise level sigma, for one slot
 * (host buffers; blocks until done). */
mkb_status mkb_dit_step(mkb_dit* d, const float* latents, float sigma, float* out, int slot);

/* n samples in one pass (batch): sample i uses slots[i], latents + i*N*64 and sigmas[i]; velocities to out + i*N*64.
 * All slots need the same prompt length; ref21 also needs them at the same step count. Host buffers. */
mkb_status mkb_dit_step_batch(mkb_dit* d, int n, const int* slots, const float* latents, const float* sigmas,
                              float* out);

/* The same on device buffers (latents_dev / out_dev [n][N][64] fp32), enqueued on `stream` without a host sync
 * (stream NULL: the handle's own non-blocking stream, which does not order with the legacy default stream). */
mkb_status mkb_dit_step_batch_dev(mkb_dit* d, int n, const int* slots, const float* latents_dev, const float* sigmas,
                                  float* out_dev, void* stream);

/* One guided Euler step of a generation (Engine::generate's loop body, engine.cpp:471-506): the cond (slot 0) and
 * uncond (slot 1) predictions in one batched pass, v = v_u + guidance (v_c - v_u), latents += (sigma_next - sigma) v.
 * latents [N][64] host fp32, updated in place. */
mkb_status mkb_dit_step_cfg(mkb_dit* d, float* latents, float sigma, float sigma_next, float guidance);

/* The device-buffer form of mkb_dit_step_cfg for n_images images at once (2 * n_images samples; image i uses slots
 * 2i and 2i+1): latents_dev [n_images][N][64] updated in place on `stream`. */
mkb_status mkb_dit_step_cfg_dev(mkb_dit* d, int n_images, float* latents_dev, float sigma, float sigma_next,
                                float guidance, void* stream);
/* The guided velocity of the same CFG batch, v = v_u + guidance (v_c - v_u), into v_out_dev [n_images][N][64]
 * without updating the latents: the model output for the device samplers below (engine.cpp:474-480). */
mkb_status mkb_dit_guided_velocity_dev(mkb_dit* d, int n_images, const float* latents_dev, float sigma,
                                       float guidance, float* v_out_dev, void* stream);

/* Stage probe, as the reference's probe() hooks (qwen_image.cpp:200-287): when set, step calls fn(name, layer,
 * data, count, user) with host fp32 copies of named stages ("temb", "txt_in", "img_in", "block" with the block index,
 * "norm_out"; qwen1 blocks report "block.txt" and "block.img"). NULL turns it off. Probing synchronises. */
typedef void (*mkb_probe_fn)(const char* name, int layer, const float* data, long count, void* user);
mkb_status mkb_dit_set_probe(mkb_dit* d, mkb_probe_fn fn, void* user);

/* Sequence parallelism (qwen1 variant), for one image batch spread over `world` GPUs, one handle and process per
 * GPU. No counterpart in the reference, which runs on one device. Each rank owns a contiguous
 * 1/world of every sample's joint rows (all text rows on rank 0), runs every GEMM, norm and RoPE on its rows, and the
 * ranks all-gather each block's K and V over NCCL so attention sees every key. Step calls keep their meaning: every
 * rank passes the same full latents and gets the full velocities / updated latents. Needs (S + N) divisible by
 * world, (S + N) / world a multiple of 128 and larger than S. Results equal the one-GPU step bit for bit.
 * mkb_nccl_unique_id makes the communicator id on one rank (MKB_NCCL_ID_BYTES bytes, to be sent to the others);
 * every rank then calls mkb_dit_set_sequence_parallel with it, collectively, after create and before begin. NCCL is
 * loaded at run time: the process's libnccl.so.2, or the library the environment variable MKB_NCCL_LIB names. If the
 * communicator cannot be made (MKB_ERR_CUDA) or its buffers not allocated (MKB_ERR_ALLOC), the handle is left as it
 * was, single-GPU and usable. */
#define MKB_NCCL_ID_BYTES 128
mkb_status mkb_nccl_unique_id(void* out, size_t bytes);
mkb_status mkb_dit_set_sequence_parallel(mkb_dit* d, const void* nccl_id, int rank, int world);
/* Moves the per-block K/V exchange of a sequence-parallel handle from the NCCL all-gather to peer memory (enable 1)
 * or back (0); collective, every rank with the same value, after mkb_dit_set_sequence_parallel. No counterpart in the
 * reference. Every rank exports a K/V region over CUDA IPC (the ranks must share a node, each GPU able to reach the
 * others) and maps the others'; after each block's QKV projection a copy engine pushes the rank's shard into every
 * peer's region and then raises the rank's ready flag there, and the attention starts on its own shard and waits
 * (bounded, 2 s; MKB_ERR_KERNEL on timeout) for each other shard's flag, so the transfers overlap the attention
 * instead of preceding it. The key order differs per rank, so results match the one-GPU step to rounding, no longer
 * bit for bit; all ranks still end with identical latents. Turns the head exchange (below) off. Fails with
 * MKB_ERR_CUDA on every rank if any rank cannot allocate, export or map, leaving the all-gather in place. */
mkb_status mkb_dit_sp_peer_exchange(mkb_dit* d, int enable);
/* Replaces the per-block K/V all-gather of a sequence-parallel handle by a head-parallel exchange (mode 1: NCCL,
 * mode 2: peer memory) or goes back to it (mode 0); collective, every rank with the same mode, after
 * mkb_dit_set_sequence_parallel. No counterpart in the reference. Rank r attends over all joint rows of heads
 * [r * H / world, (r + 1) * H / world): after each block's QKV projection every rank's rows of those heads reach rank
 * r, and after the attention its outputs return to the ranks that own the rows, before the output projection. A rank
 * receives 4 (world - 1) / world^2 of one step-wide activation per block against the all-gather's
 * 2 (world - 1) / world (a quarter at eight ranks). Mode 1 moves the rows by two NCCL all-to-alls per block. Mode 2
 * has the QKV and attention epilogues store them straight into the peers' memory (CUDA IPC regions; the ranks must
 * share a node, each GPU able to reach the others): each rank raises a flag in every peer after its stores, the
 * attention waits (bounded, 2 s; MKB_ERR_KERNEL on timeout) for a peer's flag before its first tile of that peer's
 * rows, and the output projection for every peer's attention. Every row sees its keys in the one-GPU order, so
 * both modes equal the one-GPU step bit for bit. Needs the head count divisible by world (MKB_ERR_INVALID
 * otherwise); turns the peer K/V exchange off; MKB_ERR_ALLOC / MKB_ERR_CUDA on every rank if any rank cannot
 * allocate, export or map, leaving the all-gather in place. */
mkb_status mkb_dit_sp_head_exchange(mkb_dit* d, int mode);
/* The rows rank `rank` of `world` owns for S text and N image tokens per sample: text_rows (S on rank 0, else 0),
 * image_rows starting at image token image_row0, and shard_rows = (S + N) / world joint rows. Host arithmetic only. */
mkb_status mkb_dit_sp_rows(int S, int N, int world, int rank, int* text_rows, int* image_rows, int* image_row0,
                           int* shard_rows);

/* Algorithmic FLOPs of one step over n samples at the current grid and prompt length (GEMMs + attention). */
double mkb_dit_step_flops(const mkb_dit* d, int n, int first_step);

/* ---------------------------------------------------------------------------------------------------------------
 * Schedule and samplers of the generation loop (host code; Engine::sigmas / generate, src/image/engine.cpp:335-506,
 * and image::ErSde, src/image/er_sde.hpp:12-27).
 * ------------------------------------------------------------------------------------------------------------- */

/* The flow-matching schedule's shift (Engine::Schedule, src/image/engine.hpp:251-256). */
typedef struct mkb_schedule {
    double base_seq, max_seq, base_shift, max_shift, terminal;
    int fixed_mu; /* nonzero: use mu instead of the token-count shift (distilled models) */
    double mu;
} mkb_schedule;

/* The reference's defaults: base 256 -> 0.5, max 4096 -> 1.15, no terminal stretch. */
void mkb_schedule_default(mkb_schedule* s);

/* Engine::sigmas (engine.cpp:347-365): steps noise levels for `tokens` latent tokens, then 0; out has steps + 1
 * entries. sched NULL: the defaults. */
mkb_status mkb_sigmas(const mkb_schedule* sched, uint32_t steps, uint32_t tokens, float* out);

/* Engine::top_sigma (engine.cpp:341-345): where ER-SDE starts for a flow model instead of 1. */
float mkb_top_sigma(const mkb_schedule* sched, uint32_t tokens);

/* x += (sigma_next - sigma) * (v_u + guidance * (v_c - v_u)) on host arrays of n floats (v_uncond NULL: no
 * guidance): the guided Euler update of engine.cpp:475-480, 500-503. */
void mkb_guided_euler(float* x, const float* v_cond, const float* v_uncond, float guidance, float sigma,
                      float sigma_next, long n);

/* ER-SDE (image::ErSde): the three-stage extended reverse-time SDE solver. */
typedef struct mkb_er_sde mkb_er_sde;
/* sigmas: the schedule ending at 0 (n entries); flow: latents are (1 - s) image + s noise; top: a flow model's
 * first level in place of 1 (ErSde::ErSde, er_sde.cpp:17-25). */
mkb_status mkb_er_sde_create(const float* sigmas, int n, int flow, float top, mkb_er_sde** out);
void mkb_er_sde_destroy(mkb_er_sde* e);
/* The level step i runs the model at (ErSde::sigma). */
float mkb_er_sde_sigma(const mkb_er_sde* e, int i);
/* x (n floats) from level i to i + 1 given the model's image estimate `denoised` and unit-normal noise scaled by
 * s_noise (ErSde::step, er_sde.cpp:27-74). */
mkb_status mkb_er_sde_step(mkb_er_sde* e, int i, float* x, const float* denoised, const float* noise, long n,
                           float s_noise);

/* ---- Samplers on the device (the updates of Engine::generate's loop, src/image/engine.cpp:471-506, on device
 * latents; stream-ordered, no host round trip). Noise is the counter-based generator's stream `noise_key`: element j
 * of a step draws element noise_offset + j (splitmix64 + Box-Muller, the generator of the synthetic inputs), so a run
 * is reproducible from (key, offsets). The reference draws from its host RNG; only the distribution matches. */

/* out = v_uncond + guidance (v_cond - v_uncond), n floats (engine.cpp:476-480). */
mkb_status mkb_cfg_combine_dev(float* out, const float* v_cond, const float* v_uncond, float guidance, long n,
                               void* stream);
/* x += a v, n floats: the plain Euler update with a = sigma_next - sigma (engine.cpp:500-503). */
mkb_status mkb_axpy_dev(float* x, const float* v, float a, long n, void* stream);
/* Euler-ancestral (engine.cpp:492-499): up = min(s', sqrt(s'^2 (s^2 - s'^2) / s^2)), x += (sqrt(s'^2 - up^2) - s) v,
 * then + up * noise. s = sigma > 0, s' = sigma_next in [0, s]. */
mkb_status mkb_euler_ancestral_dev(float* x, const float* v, float sigma, float sigma_next, uint64_t noise_key,
                                   uint64_t noise_offset, long n, void* stream);
/* ER-SDE step i on device latents x, v the guided model output: the image estimate x - sigma_i v
 * (engine.cpp:483-487) enters mkb_er_sde_step's update with the same coefficients. state_dev: 2n floats the caller
 * keeps for one run (previous estimate, previous difference); the run's steps go 0, 1, 2, ... (step 0 starts a new
 * run). Noise is drawn when sigma_{i+1} > 0 and s_noise > 0. */
mkb_status mkb_er_sde_step_dev(mkb_er_sde* e, int i, float* x, const float* v, float* state_dev, uint64_t noise_key,
                               uint64_t noise_offset, long n, float s_noise, void* stream);

/* ---------------------------------------------------------------------------------------------------------------
 * The SDXL UNet (Sdxl::begin / step, src/image/sdxl.cpp:672-953) and the SDXL VAE decoder (Engine::decode,
 * src/image/engine.cpp:862-954 with the AutoencoderKL layout). Latents cross the boundary as the reference's tokens:
 * [gh * gw][16], each a 2x2 patch of the 4-channel latent image (sdxl.cpp:80-87).
 * Weights are named by block position ("in4.res.conv1.w", "out3.attn.b1.ff1.w", ...; mkb_unet_weight_info), a
 * 3x3 convolution is [Cout][3][3][Cin], a 1x1 one [Cout][Cin], q/k/v stacked ([3c][c]) and the GEGLU projection
 * [8c][c] (hidden rows, then gate rows) as the reference stacks them (sdxl.cpp:285-299).
 * ------------------------------------------------------------------------------------------------------------- */

typedef struct mkb_unet_config {
    int channels[3];  /* per level: 320, 640, 1280 (multiples of 64; 128 where a level has attention) */
    int depth[3];     /* transformer blocks per attention layer of each level: 0, 2, 10 (the middle uses depth[2]) */
    int layers;       /* residual blocks per down level (2); up levels have layers + 1 */
    int context_dim;  /* 2048 */
    int pooled_dim;   /* 1280 */
    int max_batch;    /* samples per step (sample i uses slot slot0 + i) */
    int max_gh, max_gw; /* token grid maxima (the latent image is 2gh x 2gw; gw a multiple of 16, gh even) */
    int max_context;  /* context rows (77) */
    int slots;        /* text conditionings kept (2 = cond / uncond) */
} mkb_unet_config;

typedef struct mkb_unet mkb_unet;
mkb_status mkb_unet_create(const mkb_unet_config* cfg, mkb_unet** out);
void mkb_unet_destroy(mkb_unet* u);
mkb_status mkb_unet_init_random(mkb_unet* u, uint64_t seed, float std);
int mkb_unet_weight_count(const mkb_unet* u);
/* Name and logical shape (ndim 1, 2 or 4 of dims[4]) of weight i. */
mkb_status mkb_unet_weight_info(const mkb_unet* u, int i, const char** name, long* dims, int* ndim);
mkb_status mkb_unet_weight_read(mkb_unet* u, const char* name, float* host);
mkb_status mkb_unet_weight_write(mkb_unet* u, const char* name, const float* host);
/* Sdxl::begin: the context [S][context_dim] and pooled state [pooled_dim] of one prompt on a gh x gw token grid:
 * the added conditioning and every transformer block's cross-attention K/V, kept per slot. */
mkb_status mkb_unet_begin(mkb_unet* u, const float* context, int S, const float* pooled, int gh, int gw, int slot);
/* Sdxl::step: predicted noise tokens for latent tokens at noise level sigma (host buffers). */
mkb_status mkb_unet_step(mkb_unet* u, const float* latents, float sigma, float* out, int slot);
/* n samples in one pass, sample i on slot slot0 + i (host / device buffers). */
mkb_status mkb_unet_step_batch(mkb_unet* u, int n, int slot0, const float* latents, const float* sigmas, float* out);
mkb_status mkb_unet_step_batch_dev(mkb_unet* u, int n, int slot0, const float* latents_dev, const float* sigmas,
                                   float* out_dev, void* stream);
/* One guided Euler step of a generation: cond (slot 0) and uncond (slot 1) in one batched pass, then
 * latents += (sigma_next - sigma) (e_u + guidance (e_c - e_u)) on the device (engine.cpp:471-506). */
mkb_status mkb_unet_step_cfg_dev(mkb_unet* u, float* latents_dev, float sigma, float sigma_next, float guidance,
                                 void* stream);
mkb_status mkb_unet_set_probe(mkb_unet* u, mkb_probe_fn fn, void* user);
double mkb_unet_step_flops(const mkb_unet* u, int n);
/* Sdxl::sigmas (sdxl.cpp:653-670): steps levels then 0 (out has steps + 1 entries), and Sdxl::timestep (:643-651). */
mkb_status mkb_sdxl_sigmas(uint32_t steps, float* out);
int mkb_sdxl_timestep(float sigma);

typedef struct mkb_vae_config {
    int channels[4]; /* block widths from the output side: 128, 256, 512, 512 (multiples of 128) */
    int layers;      /* 2: each up level has layers + 1 residual blocks */
    int latent;      /* latent channels: 4 (SDXL) or 16 (the Qwen-Image-size token of 64 values) */
    float scale;     /* by default latents are tokens / scale (0.13025 for SDXL); see mkb_vae_set_latent_stats */
    int max_gh, max_gw;
} mkb_vae_config;

typedef struct mkb_vae mkb_vae;
mkb_status mkb_vae_create(const mkb_vae_config* cfg, mkb_vae** out);
void mkb_vae_destroy(mkb_vae* v);
mkb_status mkb_vae_init_random(mkb_vae* v, uint64_t seed, float std);
int mkb_vae_weight_count(const mkb_vae* v);
mkb_status mkb_vae_weight_info(const mkb_vae* v, int i, const char** name, long* dims, int* ndim);
mkb_status mkb_vae_weight_read(mkb_vae* v, const char* name, float* host);
mkb_status mkb_vae_weight_write(mkb_vae* v, const char* name, const float* host);
/* The UNet's and the VAE decoder's weights from safetensors checkpoints (F32 / F16 / BF16): the UNet under the
 * original checkpoint names, optionally prefixed "model.diffusion_model." (Sdxl::load_unet, src/image/sdxl.cpp:
 * 238-362); the VAE under the Diffusers names or the original AutoencoderKL ones, optionally prefixed
 * "first_stage_model." or "vae." (engine.cpp:92-118, 590-640). Convolutions are converted from [out][in][ky][kx],
 * q/k/v and cross k/v rows stacked. Other tensors in the files (a single-file checkpoint's text encoders) are ignored.
 * strict != 0: a weight the files lack is an error. *loaded (optional) counts the weights written. */
mkb_status mkb_unet_load_safetensors(mkb_unet* u, const char* const* paths, int n_paths, int strict, int* loaded);
mkb_status mkb_vae_load_safetensors(mkb_vae* v, const char* const* paths, int n_paths, int strict, int* loaded);
/* LoRA on the UNet (Sdxl::lora_target, src/image/sdxl.cpp:385-417): the transformers' proj_in / proj_out, attn1
 * to_q / to_k / to_v / to_out.0, attn2 (the same), ff.net.0.proj and ff.net.2, by checkpoint module name
 * ("input_blocks.4.1.transformer_blocks.0.attn1.to_q"; '_' and '.' compare equal, as the reference's lora_key does).
 * mkb_unet_weight_lora_rows merges into rows of a named matrix of the table; the file form reads pairs as
 * mkb_dit_load_lora does ("lora_unet_" prefixes dropped). */
mkb_status mkb_unet_weight_lora_rows(mkb_unet* u, const char* name, long row0, long rows, const float* A,
                                     const float* B, int rank, float scale);
mkb_status mkb_unet_lora_merge(mkb_unet* u, const char* module, const float* A, const float* B, int rank,
                               int in_features, int out_features, float scale);
mkb_status mkb_unet_load_lora(mkb_unet* u, const char* path, float scale, int* merged);
/* Engine::decode: tokens [gh * gw][4 * latent] to RGBA [16 gh][16 gw][4] in [-1, 1] (alpha 1), host / device
 * buffers. */
mkb_status mkb_vae_decode(mkb_vae* v, const float* latents, int gh, int gw, float* rgba);
mkb_status mkb_vae_decode_dev(mkb_vae* v, const float* latents_dev, int gh, int gw, float* rgba_dev, void* stream);
mkb_status mkb_vae_set_probe(mkb_vae* v, mkb_probe_fn fn, void* user);
double mkb_vae_decode_flops(const mkb_vae* v, int gh, int gw);
/* The latent statistics the decoder undoes first: token value i (of 4 * latent: channel c, patch row py, column px
 * at i = (c * 2 + py) * 2 + px) enters as v * std[i] + mean[i], the reference's per-value latents_mean /
 * latents_std (Engine::decode, engine.cpp:890-898; a 16-channel VAE's config.json statistics repeated over the 2x2
 * patch, or the batch-norm statistics of a packed-latent VAE). n = 4 * latent. Replaces the scale's default of
 * mean 0, std 1 / scale. */
mkb_status mkb_vae_set_latent_stats(mkb_vae* v, const float* mean, const float* std, int n);

/* ---------------------------------------------------------------------------------------------------------------
 * SDXL's text encoders: the text side of Sdxl (src/image/sdxl.hpp:46 encode_clip, and :30 prompt_embeddings, the
 * override of engine.hpp:161). The tokenizer (image::ClipTokenizer) stays with the caller: these take its token ids.
 * ------------------------------------------------------------------------------------------------------------- */

typedef struct mkb_clip_config {
    int which;      /* 0: CLIP ViT-L (quick GELU; the output is its second to last layer's states); 1: OpenCLIP bigG
                       (erf GELU; also the pooled state: the final state at the first end token, ln_final, times the
                       1280-wide text projection) */
    int width;      /* E: 768 / 1280, a multiple of 128, heads of 64 */
    int heads;      /* E / 64 */
    int layers;     /* 12 / 32 */
    int ffn;        /* 3072 / 5120 */
    int vocab;      /* 49408 */
    int max_chunks; /* 77-token chunks one encode call takes */
} mkb_clip_config;

typedef struct mkb_clip mkb_clip;
mkb_status mkb_clip_create(const mkb_clip_config* cfg, mkb_clip** out);
void mkb_clip_destroy(mkb_clip* c);
mkb_status mkb_clip_init_random(mkb_clip* c, uint64_t seed, float std);
/* The weight table: "tok" [vocab][E] and "pos" [77][E] (fp32: the checkpoint's F16 embeddings kept exactly),
 * per layer "lN.ln1.w/b", "lN.qkv.w" [3E][E] (q, k, v rows), "lN.qkv.b", "lN.o.w/b", "lN.ln2.w/b", "lN.fc1.w"
 * [F][E], "lN.fc1.b", "lN.fc2.w" [E][F], "lN.fc2.b"; bigG also "lnf.w/b" and "proj" [E][1280] as stored. */
int mkb_clip_weight_count(const mkb_clip* c);
mkb_status mkb_clip_weight_info(const mkb_clip* c, int i, const char** name, long* dims, int* ndim);
mkb_status mkb_clip_weight_read(mkb_clip* c, const char* name, float* host);
mkb_status mkb_clip_weight_write(mkb_clip* c, const char* name, const float* host);
/* Weights from an SDXL checkpoint (Sdxl::load_clip, sdxl.cpp:154-237): ViT-L under
 * "conditioner.embedders.0.transformer.text_model." (HF CLIPTextModel names, q / k / v stacked), bigG under
 * "conditioner.embedders.1.model." (OpenCLIP names: in_proj, c_fc, c_proj, ln_final, text_projection); the prefixes
 * may also be absent. strict and loaded as for mkb_vae_load_safetensors. */
mkb_status mkb_clip_load_safetensors(mkb_clip* c, const char* const* paths, int n_paths, int strict, int* loaded);
mkb_status mkb_clip_set_probe(mkb_clip* c, mkb_probe_fn fn, void* user);
/* Sdxl::encode_clip (sdxl.cpp:459-546) for `chunks` chunks of 77 token ids (host [chunks][77]): hidden (host,
 * [chunks * 77][E]) the second to last layer's states; pooled (host [chunks][1280], bigG only, may be NULL) each
 * chunk's pooled state (a bigG chunk must hold the end token 49407). Causal attention in heads of 64; projections
 * take their inputs split into bf16 parts as the reference's do. Ids out of range are MKB_ERR_INVALID. */
mkb_status mkb_clip_encode(mkb_clip* c, const int32_t* ids, int chunks, float* hidden, float* pooled);
/* Sdxl::prompt_embeddings after tokenization (sdxl.cpp:599-639): chunks of ids for each encoder (ViT-L padded with
 * the end token, bigG with 0, as Sdxl::chunks pads them) and per-token weights (host [chunks][77], NULL = all 1) to
 * context (host [chunks * 77][E_L + E_G], ViT-L's then bigG's states per token; a token of weight w != 1 gets
 * (z - e) w + e with e the empty prompt's states at its position) and pooled (host [1280], the first chunk's). */
mkb_status mkb_sdxl_prompt_embeddings(mkb_clip* l, mkb_clip* g, const int32_t* ids_l, const int32_t* ids_g,
                                      const float* weights, int chunks, float* context, float* pooled);

/* Image output (host code, no device needed). mkb_to_rgba8: RGBA floats in [-1, 1] to 8-bit samples, x / 2 + 1/2
 * clamped, times 255, rounded to nearest (the reference's to_rgba8, src/image/png.hpp:13-14, png.cpp:148-156).
 * mkb_png_encode: a PNG of 8-bit RGBA [height][width][4] (colour type 6), or with rgb != 0 of its RGB samples (colour
 * type 2), written with this library's own encoder (stored deflate blocks; the reference's encode_png,
 * png.hpp:15-17, uses Apple's ImageIO). With out == NULL only *size is set; otherwise capacity must hold *size
 * bytes. */
mkb_status mkb_to_rgba8(const float* rgba, size_t count, uint8_t* out);
mkb_status mkb_png_encode(const uint8_t* rgba8, uint32_t width, uint32_t height, int rgb, uint8_t* out,
                          size_t capacity, size_t* size);

/* The status word kernels write their error bits to (device memory owned by the library; 0 = no error). Reads and
 * clears it: returns MKB_OK, or MKB_ERR_KERNEL with the bits in *bits. Synchronises the device. */
mkb_status mkb_check_kernels(uint32_t* bits);

/* Failure-path self-test of the bounded waits (no counterpart in the reference, whose Metal command buffers have no
 * kernel-side timeouts). Launches the fp32-output projection of mkb_proj (y = x * w^T, tile width 128, one CTA per
 * SM) with the first shared-memory stage of CTA 0 never loaded: that CTA's MMA warp waits for it until its 2 s
 * limit, marks the status word and the CTA's abort flag, every role drains what it issued (another bounded wait on
 * the withheld stage) and the kernel returns after about 4 s. The other CTAs finish their tiles normally; y is left
 * incomplete. Afterwards mkb_check_kernels returns MKB_ERR_KERNEL with bit 0 (a stage that never filled) or bit 1
 * (a stage never released: the producer's own wait, whichever gives up first) and bit 4 (the drain of the withheld
 * load) set, and the context stays usable. For tests of error detection; nothing else calls it. */
mkb_status mkb_selftest_stalled_gemm(const void* x, long ldx, const void* w, long ldw, float* y, long ldy, int M,
                                     int N, int K, void* stream);

/* Failure-path self-test of the head exchange's wait for its peers (mkb_dit_sp_head_exchange mode 2; no counterpart
 * in the reference): launches the wait that holds a rank's output projection until every flag in `flags` (n device
 * words, the rank's own at index `self` skipped) has reached *value (a device word). A flag that stays below runs
 * out the bounded 2 s wait; mkb_check_kernels then returns MKB_ERR_KERNEL with bit 0x100 and the context stays
 * usable. For tests of error detection; nothing else calls it. */
mkb_status mkb_selftest_peer_wait(const unsigned long long* flags, int n, int self, const unsigned long long* value,
                                  void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MKB_IMAGE_H */
