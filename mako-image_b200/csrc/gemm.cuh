// Persistent tcgen05 GEMM for sm_100a: Y[M][N] = X[M][K] * W[N][K]^T with bf16 operands, fp32 accumulation in
// tensor memory and fused epilogues. This replaces the runtime's `proj()` matrix product that the reference calls
// for every projection of the denoiser (src/image/qwen_image.cpp:196-288 and src/image/sdxl.cpp:763-794), together
// with the element-wise kernels that follow it there: bias, activation (`gelu_tanh`, `silu`, `swiglu_rows`), the
// gated residual add (`gate_add`, src/kernels/image.metal:56-65) and the per-head RMSNorm + RoPE into the attention
// layout (`heads_norm_half` / `heads_half`, src/image/qwen_image.cpp:226-250).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace mkb {

enum class Epi : int {
    kBF16 = 0,    // out_bf16[row][col] = act(acc + bias)
    kF32 = 1,     // out_f32[row][col]  = act(acc + bias)
    kResid = 2,   // resid[row][col] += g(gate[b][col]) * (acc + bias), fp32 residual stream
    kQkv = 3,     // q/k: RMSNorm per 128-wide head, weight, RoPE; v: as is; bf16 into [B][H][L][128]
    kSwiGLU = 4,  // columns come in 128-wide (first | second) pairs: out_bf16[row][col/2] = glu(first, second)
    kAdd = 5,     // out[row][col] = acc + bias + addvec[sample][col] + resid[row][col], fp32 or bf16 out
    kHeads = 6,   // scatter into head-major [B][H][L][head_dim] bf16 (no norm): the layout of q/k/v
};

// kSwiGLU variants: the reference's SwiGLU (gate rows first) and SDXL's GEGLU (hidden rows first, erf GELU on the
// gate half).
enum Glu : int { kGluSilu = 0, kGluGelu = 1 };

// Epilogue activations: GELU (tanh form), SiLU, quick GELU x sigmoid(1.702 x) and the erf GELU (the CLIP text
// encoders' fc1, sdxl.cpp:508).
enum Act : int { kActNone = 0, kActGeluTanh = 1, kActSilu = 2, kActQuickGelu = 3, kActGeluErf = 4 };

struct GemmArgs {
    int M = 0, N = 0, K = 0;
    const float* bias = nullptr;  // [N] or null
    int act = kActNone;
    // kBF16 / kF32 / kSwiGLU output
    void* out = nullptr;
    long ldo = 0;
    // kResid
    float* resid = nullptr;
    long ldr = 0;
    const float* gate = nullptr;  // gate of sample b at gate + b * gate_bstride
    long gate_bstride = 0;
    int tanh_gate = 0;            // x += tanh(g) * y (the reference's gate_add) instead of x += g * y
    int gate_split = 0;           // rows whose index within their sample is < gate_split use gate + gate_alt_off
    long gate_alt_off = 0;        //   (the reference's text rows take modulation row 1)
    // rows -> (sample, position): sample = row / seg_rows, position = seg_off + row % seg_rows
    int seg_rows = 1 << 30;
    int seg_off = 0;
    // kQkv
    __nv_bfloat16* qh = nullptr;
    __nv_bfloat16* kh = nullptr;
    __nv_bfloat16* vh = nullptr;
    const float* norm_q = nullptr;  // [128]
    const float* norm_k = nullptr;  // [128]
    const float* rope = nullptr;    // [L][64][2] (cos, sin) per joint position, or null for no rotation
    int D = 0;                      // width of each of q, k, v (heads * head_dim)
    int L = 0;                      // joint sequence length of the head layout
    // kQkv: heads in groups of head_group (0: one group, the layout above). Head h of group g = h / head_group goes
    // to group_dst[g] + which * group_chunk + ((sample * head_group + h % head_group) * L + position) * 128 (which:
    // 0 q, 1 k, 2 v); group_dst is a device array of one base per group: the spans of the head-parallel exchange,
    // in this GPU's memory or mapped from the peer that attends over those heads.
    int head_group = 0;
    long group_chunk = 0;
    __nv_bfloat16* const* group_dst = nullptr;
    float eps = 1e-6f;
    int head_dim = 128;             // kHeads: 64 or 128
    int part0 = 0;                  // kHeads: the first column block goes to q (0), k (1) or v (2)
    // kSwiGLU
    int glu = kGluSilu;
    // kAdd
    const float* addvec = nullptr;  // per-sample vector (sample = row / seg_rows), stride addvec_stride
    long addvec_stride = 0;
    const float* add_resid = nullptr;  // fp32 [row][col] rows ld_add_resid apart (may alias out)
    long ld_add_resid = 0;
    int out_f32 = 1;
    // Set by the prepare functions: how a kAdd fp32 or kResid tile leaves the SM. 0: each epilogue thread stores
    // its row; otherwise 32-column boxes staged in shared memory go out with TMA: 1 store, 2 reduce-add into the
    // output (the residual is the output itself; always so for kResid), 3 residual box loaded with TMA, added,
    // stored.
    int out_mode = 0;
    // 3x3 / 1x1 convolution as an implicit GEMM (k_gemm's conv mode): the A operand is the channels-last bf16
    // input [B][conv_hi][conv_wi][conv_c], the output pixel grid [B][conv_ho][conv_wo] is cut into tiles of
    // conv_th x conv_tw pixels (128 rows), and K = conv_taps * conv_c runs tap by tap.
    int conv_hi = 0, conv_wi = 0, conv_c = 0, conv_ho = 0, conv_wo = 0;
    int conv_stride = 1, conv_taps = 0, conv_pad = 0, conv_tw = 16, conv_th = 8, conv_b = 0;
    // A convolution's kAdd epilogue with fp32 boxes can also leave the GroupNorm statistics of its output (the
    // values it stores, after bias and residual): per image, group of gn_cpg channels (4, 8 or 16) and 32 pixels,
    // float4 (count, mean, M2, 0) at gn_part[(image * (N / gn_cpg) + group) * gn_chunks + chunk], where chunk =
    // (the tile's index within its image) * 4 + the tile's 32-pixel quarter. conv_prepare sets gn_chunks.
    float4* gn_part = nullptr;
    int gn_cpg = 0;
    int gn_chunks = 0;
    uint32_t* status = nullptr;     // error bits (kErr*), may be null
};

// The kernel's parameters: one or two problems of the same epilogue kind and tile width run by one persistent
// launch (problem 0's tiles first, problem 1's filling the tail).
struct GemmParams {
    CUtensorMap ta[2];
    CUtensorMap tb[2];
    CUtensorMap to[2];  // output boxes (out_mode != 0)
    CUtensorMap tr[2];  // residual boxes (out_mode 3)
    GemmArgs a[2];
    int nprob = 1;
    int tiles0 = 0;
    // Failure-path testing only (mkb_selftest_stalled_gemm): the 1-CTA kernel's CTA 0 withholds the TMA load of its
    // first stage, so the MMA warp's bounded wait on that stage runs out and the kernel takes its error exit.
    int test_stall = 0;
};

// A prepared launch: tensor maps and arguments are built once (buffers are fixed), then launched any number of
// times, also inside CUDA graph capture.
struct GemmOp {
    GemmParams p;
    Epi epi = Epi::kBF16;
    int bn = 256;
    int grid = 0;
    bool conv = false;
    bool pair = false;  // CTA-pair (cta_group::2) kernel: 256-row tiles shared by two SMs
    bool ready = false;
    const void* w_ptr[2] = {nullptr, nullptr};  // W operands and their row strides (to re-encode W's maps)
    long ldw[2] = {0, 0};
};

// Builds a GemmOp. X: [M][K] bf16 rows `ldx` elements apart; W: [N][K] bf16 rows `ldw` apart. Returns false with a
// message in *err on unsupported shapes or misaligned pointers.
bool gemm_prepare(GemmOp& op, Epi epi, const void* X, long ldx, const void* W, long ldw, const GemmArgs& args,
                  int bn, const char** err);
// Switches a prepared (non-convolution) GEMM to the CTA-pair kernel: 256-row tiles, each SM loading half of the W
// tile. Needs the tile width >= 128. Call after adding any second problem.
bool gemm_use_pairs(GemmOp& op, const char** err);

// The tile (width 64, 128, 160, 192 or 256; 1-CTA or, when allowed, CTA pair) with the shortest estimated makespan
// for an M x N output on this GPU's SMs; only_bn restricts the width. N must be a multiple of 32.
struct GemmTile {
    int bn;
    bool pairs;
};
GemmTile gemm_pick_tile(long M, int N, bool allow_pairs, int only_bn = 0);
// The width alone, for the 1-CTA kernel or (pairs) the CTA-pair kernel.
int gemm_pick_bn(long M, int N, bool pairs = false);
// Adds a second problem (same epilogue kind and tile width; X [M][K], W [N][K]) to a prepared GEMM.
bool gemm_add_problem(GemmOp& op, const void* X, long ldx, const void* W, long ldw, const GemmArgs& args,
                      const char** err);
cudaError_t gemm_launch(const GemmOp& op, cudaStream_t stream);

// Chunks per image of a convolution's GroupNorm statistics (GemmArgs::gn_part) at output size Ho x Wo.
int conv_gn_chunks(int Ho, int Wo);

// Builds a convolution as an implicit GEMM: X is the channels-last bf16 input [B][Hi][Wi][C] (C a multiple of 64),
// W the weights [Cout][taps][C] (taps 9 = 3x3 with padding 1, or 1), stride 1 or 2. args.M / N / K are filled in;
// the output pixel of tile row r is written at row (b * Ho + y) * Wo + x of the epilogue's output.
bool conv_prepare(GemmOp& op, Epi epi, const void* X, int B, int Hi, int Wi, int C, const void* W, int Cout,
                  int taps, int stride, const GemmArgs& args, int bn, const char** err);

int num_sms();

// Encodes a 2-D bf16 tensor map with the 128-byte swizzle: inner (contiguous) extent `inner`, `outer` rows
// `row_bytes` apart, box `box_inner` x `box_outer`.
bool make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                       uint32_t box_inner, uint32_t box_outer, const char** err);

}  // namespace mkb
