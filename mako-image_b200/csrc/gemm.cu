// Persistent warp-specialised tcgen05 GEMM (see gemm.cuh for what it replaces in the reference).
//
// One CTA per SM walks a grouped tile order. Warp 0 streams 128x64 X tiles and BNx64 W tiles into a ring of
// shared-memory stages with TMA (128-byte swizzle); warp 1 issues tcgen05.mma 128xBNx16 into one of two tensor-memory
// accumulators; warps 2-5 drain the other accumulator through the fused epilogue while the next tile accumulates.
// tcgen05.ld's 32x32b shape gives each epilogue thread one output row, so row-wise epilogue maths (per-head RMSNorm,
// RoPE pairs, SwiGLU pairs) needs no shuffles. The add, gated-residual and plain bf16 epilogues hand their rows to
// TMA instead of storing them thread by thread: each thread writes its row of a 128-byte-swizzled shared-memory box
// and one thread issues a tensor store, or a reduce-add into the residual stream.
#include "gemm.cuh"
#include "sm100.cuh"
#include "common.cuh"
#include "launch.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdio>
#include <cstdlib>
#include <mutex>

namespace mkb {

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kThreads = 192;

// The add epilogue's staging after the stages: two TMA boxes of 32 fp32 columns x 128 rows, then the current tile's
// bias (at most 256 floats).
constexpr int kEpiBox = 128 * 32 * 4;
constexpr int kBiasBytes = 256 * 4;
constexpr bool epi_tma(Epi e) { return e == Epi::kAdd || e == Epi::kResid || e == Epi::kBF16; }
// The QKV epilogue's staging: per epilogue warp one head of its 32 rows (32 x 256 bytes), so that the rows leave as
// whole 256-byte rows (coalesced; into another GPU's memory under the head-parallel exchange) rather than as
// 16-byte pieces 256 bytes apart.
constexpr int kQkvStage = 32 * 128 * 2;
constexpr int epi_staging(Epi e)
{
    return epi_tma(e) ? 2 * kEpiBox + kBiasBytes : e == Epi::kQkv ? 4 * kQkvStage : 0;
}

// Stages: up to 8 within 200 KB, fewer where the epilogue's staging would not fit beside them in 227 KB.
constexpr int stages_for(int stage_bytes, int staging)
{
    const int by_budget = (200 * 1024) / stage_bytes > 8 ? 8 : (200 * 1024) / stage_bytes;
    const int fit = (227 * 1024 - 1024 - 256 - staging) / stage_bytes;
    return by_budget < fit ? by_budget : fit;
}

template <int BN, int STG = 0>
struct Cfg {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = BN * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = stages_for(kStageBytes, STG);
    static constexpr int kTmemCols = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    static constexpr int kStaging = STG;
    static constexpr int kBarBytes = 256;
    static constexpr int kSmem = 1024 + kStages * kStageBytes + STG + kBarBytes;
    static_assert(kStageBytes % 1024 == 0, "stages and staging boxes must stay 1024-byte aligned");
};

// Per-CTA shared memory of the 2-SM kernel: the CTA's 128 rows of A and half (BN / 2 rows) of B per stage.
template <int BN, int STG = 0>
struct Cfg2 {
    static constexpr int kABytes = kBM * kBK * 2;
    static constexpr int kBBytes = (BN / 2) * kBK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStages = stages_for(kStageBytes, STG);
    static constexpr int kTmemCols = 2 * BN <= 256 ? 256 : 512;
    static constexpr int kStaging = STG;
    static constexpr int kSmem = 1024 + kStages * kStageBytes + STG + 256;
    static_assert(kStageBytes % 1024 == 0, "stages and staging boxes must stay 1024-byte aligned");
};

#ifndef MKB_TILE_GROUP
#define MKB_TILE_GROUP 8  // M-tiles per raster group: concurrent tiles share X and W panels in L2
#endif

__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int& mb, int& nb)
{
    constexpr int G = MKB_TILE_GROUP;
    const int per_group = G * num_n;
    const int group = tile / per_group;
    const int first_m = group * G;
    const int gsize = min(num_m - first_m, G);
    const int t = tile - group * per_group;
    mb = first_m + t % gsize;
    nb = t / gsize;
}

// tanh on the SFU (tanh.approx.f32, relative error ~2^-11): below the bf16 rounding of every output it feeds.
__device__ __forceinline__ float tanh_fast(float x)
{
    float y;
    asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ float gelu_tanh(float x)
{
    const float k0 = 0.7978845608028654f, k1 = 0.044715f;
    return 0.5f * x * (1.0f + tanh_fast(k0 * (x + k1 * x * x * x)));
}

__device__ __forceinline__ float silu(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ float quick_gelu(float x) { return x / (1.0f + __expf(-1.702f * x)); }

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.7071067811865476f)); }

// The activation over a 32-column chunk. The switch sits outside the loop so the 32 independent chains interleave
// (a per-element branch serializes each SFU round trip).
__device__ __forceinline__ void apply_act32(float (&v)[32], int act)
{
    if (act == kActGeluTanh) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            v[j] = gelu_tanh(v[j]);
    } else if (act == kActSilu) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            v[j] = silu(v[j]);
    } else if (act == kActQuickGelu) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            v[j] = quick_gelu(v[j]);
    } else if (act == kActGeluErf) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            v[j] = gelu_erf(v[j]);
    }
}

// The add epilogue's threads (et = 0..127) stage each tile's bias columns [n0, n0 + BN) in shared memory (zeros past
// N or without a bias), so every 32-column chunk reads a shared-memory broadcast instead of paying its own
// first-touch L2 round trip (the UNet's and VAE's GEMMs and convolutions run one to a few tiles per CTA). The first
// tile's copy is loaded while the mainloop runs; each next tile's is loaded into registers while the current tile
// drains and stored once every thread is past its last read of the current copy. The other epilogues read the bias
// per chunk: the tile-start barrier that publishes a staged copy measured 4-10% slower on their many-tile launches.
template <int BN>
struct BiasStage {
    static constexpr int kPer = (BN + 127) / 128;  // columns per epilogue thread
    float v[kPer];
    __device__ __forceinline__ void load(const GemmArgs& a, int n0, int et)
    {
#pragma unroll
        for (int k = 0; k < kPer; ++k) {
            const int i = et + 128 * k;
            v[k] = i < BN && a.bias && n0 + i < a.N ? __ldg(a.bias + n0 + i) : 0.0f;
        }
    }
    __device__ __forceinline__ void store(float* sb, int et) const
    {
#pragma unroll
        for (int k = 0; k < kPer; ++k)
            if (et + 128 * k < BN)
                sb[et + 128 * k] = v[k];
    }
};

// Bias of columns [col0, col0 + 32) from global memory (zeros without a bias).
__device__ __forceinline__ void load_bias32g(const float* bias, int col0, float (&b)[32])
{
    if (bias) {
        const float4* p = reinterpret_cast<const float4*>(bias + col0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const float4 v = __ldg(p + j);
            b[4 * j] = v.x;
            b[4 * j + 1] = v.y;
            b[4 * j + 2] = v.z;
            b[4 * j + 3] = v.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            b[j] = 0.0f;
    }
}

// Bias of tile columns [c, c + 32) from the staged copy.
__device__ __forceinline__ void load_bias32(const float* sb, int c, float (&b)[32])
{
    const float4* p = reinterpret_cast<const float4*>(sb + c);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const float4 v = p[j];
        b[4 * j] = v.x;
        b[4 * j + 1] = v.y;
        b[4 * j + 2] = v.z;
        b[4 * j + 3] = v.w;
    }
}

__device__ __forceinline__ void store_bf16x32(__nv_bfloat16* dst, const float (&v)[32])
{
    uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
    for (int j = 0; j < 4; ++j)
        d[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                          pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
}

// The epilogue of one tile for one thread (one row). t_row: TMEM address of this row's accumulator, column 0.
template <int BN, Epi EPI>
__device__ __forceinline__ void epilogue(const GemmArgs& a, uint32_t t_row, int row, bool row_ok, int n0,
                                         const float* sb, uint8_t* stg = nullptr)
{
    if constexpr (EPI == Epi::kBF16 || EPI == Epi::kF32 || EPI == Epi::kResid || EPI == Epi::kAdd) {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tmem_ld32(t_row + c, r);
            tmem_wait_ld();
            const int col0 = n0 + c;
            if (!row_ok || col0 >= a.N)
                continue;
            float b[32];
            if constexpr (EPI == Epi::kAdd || EPI == Epi::kResid)
                load_bias32(sb, c, b);
            else
                load_bias32g(a.bias, col0, b);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
                v[j] = __uint_as_float(r[j]) + b[j];
            if constexpr (EPI == Epi::kBF16) {
                apply_act32(v, a.act);
                store_bf16x32(static_cast<__nv_bfloat16*>(a.out) + long(row) * a.ldo + col0, v);
            } else if constexpr (EPI == Epi::kF32) {
                apply_act32(v, a.act);
                float4* d = reinterpret_cast<float4*>(static_cast<float*>(a.out) + long(row) * a.ldo + col0);
#pragma unroll
                for (int j = 0; j < 8; ++j)
                    d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            } else if constexpr (EPI == Epi::kAdd) {
                if (a.addvec) {
                    const float4* av =
                        reinterpret_cast<const float4*>(a.addvec + long(row / a.seg_rows) * a.addvec_stride + col0);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 t = __ldg(av + j);
                        v[4 * j] += t.x;
                        v[4 * j + 1] += t.y;
                        v[4 * j + 2] += t.z;
                        v[4 * j + 3] += t.w;
                    }
                }
                if (a.add_resid) {
                    const float4* rr = reinterpret_cast<const float4*>(a.add_resid + long(row) * a.ld_add_resid + col0);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 t = rr[j];
                        v[4 * j] += t.x;
                        v[4 * j + 1] += t.y;
                        v[4 * j + 2] += t.z;
                        v[4 * j + 3] += t.w;
                    }
                }
                if (a.out_f32) {
                    float4* d = reinterpret_cast<float4*>(static_cast<float*>(a.out) + long(row) * a.ldo + col0);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        d[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
                } else {
                    store_bf16x32(static_cast<__nv_bfloat16*>(a.out) + long(row) * a.ldo + col0, v);
                }
            } else {
                const int bsample = row / a.seg_rows;
                const int within = row - bsample * a.seg_rows;
                const float4* g4 = reinterpret_cast<const float4*>(
                    a.gate + long(bsample) * a.gate_bstride + (within < a.gate_split ? a.gate_alt_off : 0) + col0);
                float4* x4 = reinterpret_cast<float4*>(a.resid + long(row) * a.ldr + col0);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    float4 g = __ldg(g4 + j);
                    if (a.tanh_gate) {
                        g.x = tanh_fast(g.x);
                        g.y = tanh_fast(g.y);
                        g.z = tanh_fast(g.z);
                        g.w = tanh_fast(g.w);
                    }
                    float4 x = x4[j];
                    x.x += g.x * v[4 * j];
                    x.y += g.y * v[4 * j + 1];
                    x.z += g.z * v[4 * j + 2];
                    x.w += g.w * v[4 * j + 3];
                    x4[j] = x;
                }
            }
        }
    } else if constexpr (EPI == Epi::kSwiGLU) {
        // Tile columns [0, BN/2) are gates, [BN/2, BN) the matching ups; output column n0/2 + j.
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
            uint32_t rg[32], ru[32];
            tmem_ld32(t_row + c, rg);
            tmem_ld32(t_row + BN / 2 + c, ru);
            tmem_wait_ld();
            if (!row_ok || n0 + c >= a.N)
                continue;
            float bg[32], bu[32], v[32];
            load_bias32g(a.bias, n0 + c, bg);
            load_bias32g(a.bias, n0 + BN / 2 + c, bu);
            if (a.glu == kGluGelu) {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    v[j] = (__uint_as_float(rg[j]) + bg[j]) * gelu_erf(__uint_as_float(ru[j]) + bu[j]);
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    v[j] = silu(__uint_as_float(rg[j]) + bg[j]) * (__uint_as_float(ru[j]) + bu[j]);
            }
            store_bf16x32(static_cast<__nv_bfloat16*>(a.out) + long(row) * a.ldo + n0 / 2 + c, v);
        }
    } else if constexpr (EPI == Epi::kHeads) {
        // Plain scatter: 32-column chunks never straddle a head (head_dim 64 or 128).
        const int bsample = row / a.seg_rows;
        const int pos = a.seg_off + row % a.seg_rows;
        const int hd = a.head_dim, heads = a.D / hd;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tmem_ld32(t_row + c, r);
            tmem_wait_ld();
            const int col = n0 + c;
            if (!row_ok || col >= a.N)
                continue;
            float b[32], v[32];
            load_bias32g(a.bias, col, b);
#pragma unroll
            for (int j = 0; j < 32; ++j)
                v[j] = __uint_as_float(r[j]) + b[j];
            const int which = a.part0 + col / a.D;
            const int head = (col % a.D) / hd;
            __nv_bfloat16* base = which == 0 ? a.qh : which == 1 ? a.kh : a.vh;
            store_bf16x32(base + ((long(bsample) * heads + head) * a.L + pos) * hd + (col % hd), v);
        }
    } else {  // kQkv
        const int bsample = row / a.seg_rows;
        const int pos = a.seg_off + row % a.seg_rows;
        const int heads = a.D / 128;
#pragma unroll 1
        for (int hh = 0; hh < BN / 128; ++hh) {
            const int colh = n0 + hh * 128;
            const int which = colh / a.D;  // 0 q, 1 k, 2 v
            const int head = (colh % a.D) / 128;
            float rinv = 1.0f;
            if (which < 2) {
                float ss = 0.0f;
#pragma unroll 1
                for (int c = 0; c < 128; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(t_row + hh * 128 + c, r);
                    tmem_wait_ld();
                    float b[32];
                    load_bias32g(a.bias, colh + c, b);
#pragma unroll
                    for (int j = 0; j < 32; ++j) {
                        const float v = __uint_as_float(r[j]) + b[j];
                        ss += v * v;
                    }
                }
                rinv = rsqrtf(ss * (1.0f / 128.0f) + a.eps);
            }
            __nv_bfloat16* base = which == 0 ? a.qh : which == 1 ? a.kh : a.vh;
            __nv_bfloat16* dst = base + ((long(bsample) * heads + head) * a.L + pos) * 128;
            if (a.head_group > 0) {
                const int grp = head / a.head_group;
                dst = a.group_dst[grp] + which * a.group_chunk +
                      ((long(bsample) * a.head_group + head - grp * a.head_group) * a.L + pos) * 128;
            }
            if (!row_ok)
                dst = nullptr;
            const int lane = threadIdx.x & 31;
            const float* w = which == 0 ? a.norm_q : a.norm_k;
#pragma unroll 1
            for (int c = 0; c < 128; c += 32) {
                uint32_t r[32];
                tmem_ld32(t_row + hh * 128 + c, r);
                tmem_wait_ld();
                if (!row_ok)
                    continue;
                float b[32], v[32];
                load_bias32g(a.bias, colh + c, b);
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    v[j] = __uint_as_float(r[j]) + b[j];
                if (which < 2) {
                    const float4* w4 = reinterpret_cast<const float4*>(w + c);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        const float4 ww = __ldg(w4 + j);
                        v[4 * j] *= rinv * ww.x;
                        v[4 * j + 1] *= rinv * ww.y;
                        v[4 * j + 2] *= rinv * ww.z;
                        v[4 * j + 3] *= rinv * ww.w;
                    }
                    if (a.rope) {
                        const float4* cs = reinterpret_cast<const float4*>(a.rope + (long(pos) * 64 + c / 2) * 2);
#pragma unroll
                        for (int j = 0; j < 8; ++j) {  // two (cos, sin) pairs per float4
                            const float4 t = __ldg(cs + j);
                            const float x0 = v[4 * j], x1 = v[4 * j + 1], x2 = v[4 * j + 2], x3 = v[4 * j + 3];
                            v[4 * j] = x0 * t.x - x1 * t.y;
                            v[4 * j + 1] = x0 * t.y + x1 * t.x;
                            v[4 * j + 2] = x2 * t.z - x3 * t.w;
                            v[4 * j + 3] = x2 * t.w + x3 * t.z;
                        }
                    }
                }
                // This row's 64 bytes at 16-byte chunks c / 8 .. c / 8 + 3 of its 256-byte staging row, chunk j
                // placed at j ^ (row & 15) so that a warp's writes and the copy-out's reads spread over the banks.
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int j = c / 8 + k;
                    *reinterpret_cast<uint4*>(stg + lane * 256 + ((j ^ (lane & 15)) << 4)) =
                        make_uint4(pack_bf16x2(v[8 * k], v[8 * k + 1]), pack_bf16x2(v[8 * k + 2], v[8 * k + 3]),
                                   pack_bf16x2(v[8 * k + 4], v[8 * k + 5]), pack_bf16x2(v[8 * k + 6], v[8 * k + 7]));
                }
            }
            __syncwarp();
            // The warp's 32 rows of this head leave as whole rows: half a warp per 256-byte row.
#pragma unroll 4
            for (int k = 0; k < 16; ++k) {
                const int idx = k * 32 + lane, rr = idx >> 4, j = idx & 15;
                __nv_bfloat16* d = reinterpret_cast<__nv_bfloat16*>(
                    __shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(dst), rr));
                if (d)
                    *reinterpret_cast<uint4*>(d + j * 8) =
                        *reinterpret_cast<const uint4*>(stg + rr * 256 + ((j ^ (rr & 15)) << 4));
            }
            __syncwarp();
        }
    }
}

// Output tile origin of conv m-tile mb: sample, first output row and column.
__device__ __forceinline__ void conv_tile(const GemmArgs& a, int mb, int& b, int& y0, int& x0)
{
    const int tx_n = a.conv_wo / a.conv_tw, ty_n = (a.conv_ho + a.conv_th - 1) / a.conv_th;
    b = mb / (tx_n * ty_n);
    const int rem = mb - b * tx_n * ty_n;
    y0 = (rem / tx_n) * a.conv_th;
    x0 = (rem % tx_n) * a.conv_tw;
}

// The convolution's k-blocks in order: (tap, 64-channel chunk), each the tile's input window shifted by the tap
// (zero-filled outside the image: the padding). The TMA producer steps it with additions only; the tile origin is
// computed once per tile.
struct ConvWalk {
    int b = 0, x = 0, y = 0, c0 = 0;  // TMA coordinates of the current k-block's window
    int x_base = 0, y_base = 0, dx = 0;
    __device__ __forceinline__ void start(const GemmArgs& a, int mtile)
    {
        int y0, x0;
        conv_tile(a, mtile, b, y0, x0);
        x_base = x0 * a.conv_stride - a.conv_pad;
        y_base = y0 * a.conv_stride - a.conv_pad;
        x = x_base;
        y = y_base;
        c0 = 0;
        dx = 0;
    }
    __device__ __forceinline__ void next(const GemmArgs& a)
    {
        c0 += 64;
        if (c0 < a.conv_c)
            return;
        c0 = 0;
        if (a.conv_taps != 9)
            return;
        if (++dx < 3) {
            ++x;
        } else {
            dx = 0;
            x = x_base;
            ++y;
        }
    }
};

__device__ __forceinline__ int gemm_num_m(const GemmArgs& a, bool conv)
{
    return conv ? a.conv_b * (a.conv_wo / a.conv_tw) * ((a.conv_ho + a.conv_th - 1) / a.conv_th) : (a.M + kBM - 1) / kBM;
}

// 16-byte chunk j of row r of a staging box (128-byte rows, 128-byte swizzle: the chunk index XOR the row mod 8,
// which is the layout TMA reads and writes, and keeps a warp's row-per-lane accesses free of bank conflicts).
__device__ __forceinline__ float4* box_chunk(uint8_t* box, int r, int j)
{
    return reinterpret_cast<float4*>(box + r * 128 + ((j ^ (r & 7)) << 4));
}

// State of the TMA epilogue across the tiles of one CTA.
struct EpiTma {
    uint8_t* boxes;         // two kEpiBox boxes
    uint64_t* rbar;         // [2] residual-box barriers
    uint32_t chunk = 0;     // chunks issued so far: chunk & 1 is the box in use
    uint32_t rphase = 0;    // parity bit per box of its residual barrier
    uint32_t rpending = 0;  // (issuer) bit per box: a residual load for a coming chunk is in flight
    bool issuer = false;    // the one epilogue thread that issues the TMA copies
};

// (issuer, out_mode 3) Loads the residual box of tile columns [col0, col0 + 32) into box `b`.
template <bool CONV>
__device__ __forceinline__ void epi_load_resid(EpiTma& e, const CUtensorMap* tr, int b, int col0, int c1, int c2,
                                               int c3)
{
    uint8_t* box = e.boxes + b * kEpiBox;
    mbar_arrive_expect_tx(&e.rbar[b], kEpiBox);
    if constexpr (CONV)
        tma_load_4d(box, tr, &e.rbar[b], col0, c1, c2, c3);
    else
        tma_load_2d(box, tr, &e.rbar[b], col0, c1);
    e.rpending |= 1u << b;
}

// (issuer) Before a tile's accumulator is ready: starts the load of its first residual box, so the epilogue does
// not begin with an L2 round trip. The box is free once at most one store (the previous chunk's) still reads.
template <bool CONV>
__device__ __forceinline__ void epi_prefetch_tile(EpiTma& e, const GemmArgs& a, const CUtensorMap* tr, int n0,
                                                  bool tile_ok, int c1, int c2, int c3)
{
    if (a.out_mode != 3 || !tile_ok || n0 >= a.N)
        return;
    bulk_wait_read<1>();
    epi_load_resid<CONV>(e, tr, int(e.chunk & 1), n0, c1, c2, c3);
}

// (issuer) After an early exit: lets residual loads still in flight land before the CTA's shared memory goes.
__device__ __forceinline__ void epi_drain_resid(EpiTma& e, uint32_t* status)
{
    for (int b = 0; b < 2; ++b)
        if (e.rpending >> b & 1)
            mbar_wait(&e.rbar[b], (e.rphase >> b) & 1, status, kErrWaitDrain, nullptr);
}

// GroupNorm statistics of one warp's 32 rows (pixels) of a 32-column chunk of a convolution's output, for the
// 32 / CPG channel groups in the chunk. Each lane sums its row's values of every group, shifted by lane 0's first
// value of the group (shifted sums keep the variance exact to fp32 rounding for these 32 x CPG values); the lanes
// then reduce-scatter the 2 x (32 / CPG) sums in halving steps (lane bit 4 decides first, so the lane holding a
// group's shifted sum of squares is lane ^ 16 of the one holding its shifted sum) and one lane per group writes
// (count, mean, M2). Rows outside the image count nothing.
template <int CPG>
__device__ __forceinline__ void gn_warp_stats(const GemmArgs& a, const float (&v)[32], bool row_ok, int col0,
                                              int img, int chunk)
{
    constexpr int NG = 32 / CPG, V = 2 * NG, kSteps = NG == 8 ? 4 : NG == 4 ? 3 : 2;
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    float x[V], sh[NG];
    const float keep_row = row_ok ? 1.f : 0.f;
#pragma unroll
    for (int k = 0; k < NG; ++k) {
        sh[k] = __shfl_sync(full, v[k * CPG], 0);
        // Two channels per packed instruction: d = x keep - shift keep (x - shift, or 0 outside the image), then the
        // sums of d and d^2.
        const float2 kr = make_float2(keep_row, keep_row), nsk = make_float2(-sh[k] * keep_row, -sh[k] * keep_row);
        float2 s1 = make_float2(0.f, 0.f), s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < CPG; i += 2) {
            const float2 d = ffma2(make_float2(v[k * CPG + i], v[k * CPG + i + 1]), kr, nsk);
            s1 = fadd2(s1, d);
            s2 = ffma2(d, d, s2);
        }
        x[k] = s1.x + s1.y;
        x[NG + k] = s2.x + s2.y;
    }
#pragma unroll
    for (int step = 0; step < 5; ++step) {
        const int o = 16 >> step;
        const int half = V >> (step + 1);
        if (half >= 1) {
            const bool upper = (lane & o) != 0;
#pragma unroll
            for (int i = 0; i < half; ++i) {
                const float send = upper ? x[i] : x[i + half];
                const float keep = upper ? x[i + half] : x[i];
                x[i] = keep + __shfl_xor_sync(full, send, o);
            }
        } else {
            x[0] += __shfl_xor_sync(full, x[0], o);
        }
    }
    const float s2 = __shfl_xor_sync(full, x[0], 16);
    const float n = float(__popc(__ballot_sync(full, row_ok)) * CPG);
    constexpr int kLow = (1 << (5 - kSteps)) - 1;  // lane bits the final butterfly summed over
    if ((lane & 16) || (lane & kLow))
        return;
    int k = 0;
#pragma unroll
    for (int st = 1; st < kSteps; ++st)
        k += ((lane >> (4 - st)) & 1) * (V >> (st + 1));
    float shk = 0.f;
#pragma unroll
    for (int kk = 0; kk < NG; ++kk)
        shk = kk == k ? sh[kk] : shk;
    const float s1 = x[0];
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
    if (n > 0.f)
        o = make_float4(n, shk + s1 / n, fmaxf(s2 - s1 * (s1 / n), 0.f), 0.f);
    a.gn_part[(long(img) * (a.N / CPG) + col0 / CPG + k) * a.gn_chunks + chunk] = o;
}

// The fp32 epilogues through TMA. Per 32-column chunk the 128 epilogue threads (one row each, r = row within the
// tile) write their row of a staging box, then one thread stores it (out_mode 1, 3) or reduce-adds it into the
// output (out_mode 2: the output is the residual). kAdd writes acc + bias + addvec (+ the residual box, out_mode 3);
// its sums are those of the per-thread epilogue in the same order, so both paths give the same bits. kResid writes
// g * (acc + bias) with g the row's gate (tanh'd for tanh_gate), reduce-added into the residual stream: one rounding
// more than the per-thread fused multiply-add. The box is the tile's 128 rows: c1 the first row (2-D), or c1..c3 =
// x0, y0, image of a convolution's pixel tile.
template <int BN, Epi EPI, bool CONV>
__device__ __forceinline__ void epilogue_tma(const GemmArgs& a, const CUtensorMap* to, const CUtensorMap* tr,
                                             uint32_t t_row, int r, int row, bool row_ok, bool tile_ok, int n0,
                                             int c1, int c2, int c3, const float* sb, EpiTma& e,
                                             uint32_t* status, volatile int* abort)
{
    if constexpr (EPI == Epi::kBF16) {
        // bf16 output (out_mode 4): boxes of 64 columns (128 bytes a row), act(acc + bias) packed as the per-thread
        // path packs it. Tile widths are multiples of 64, so a box never reaches into a neighbouring tile.
        if constexpr (BN % 64 == 0 && !CONV) {
#pragma unroll 1
            for (int c = 0; c < BN; c += 64, ++e.chunk) {
                uint8_t* box = e.boxes + (e.chunk & 1) * kEpiBox;
                const int col0 = n0 + c;
                const bool active = tile_ok && col0 < a.N;
                if (e.issuer)
                    bulk_wait_read<1>();
                named_barrier_sync<1, 128>();
                uint32_t acc0[32], acc1[32];
                tmem_ld32(t_row + c, acc0);
                tmem_ld32(t_row + c + 32, acc1);
                tmem_wait_ld();
                if (active) {
                    float b[32], v[32];
                    uint32_t w[32];
                    load_bias32(sb, c, b);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        v[j] = __uint_as_float(acc0[j]) + b[j];
                    apply_act32(v, a.act);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        w[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
                    load_bias32(sb, c + 32, b);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        v[j] = __uint_as_float(acc1[j]) + b[j];
                    apply_act32(v, a.act);
#pragma unroll
                    for (int j = 0; j < 16; ++j)
                        w[16 + j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
#pragma unroll
                    for (int j = 0; j < 8; ++j)
                        *reinterpret_cast<uint4*>(box_chunk(box, r, j)) =
                            make_uint4(w[4 * j], w[4 * j + 1], w[4 * j + 2], w[4 * j + 3]);
                    fence_proxy_async_smem();
                }
                named_barrier_sync<1, 128>();
                if (e.issuer && active) {
                    tma_store_2d(to, box, col0, c1);
                    bulk_commit();
                }
            }
        } else if (e.issuer && status) {
            atomicOr(status, kErrShape);  // the host never prepares bf16 boxes for these tiles
        }
        return;
    }
#pragma unroll 1
    for (int c = 0; c < BN; c += 32, ++e.chunk) {
        const uint32_t buf = e.chunk & 1;
        uint8_t* box = e.boxes + buf * kEpiBox;
        const int col0 = n0 + c;
        const bool active = tile_ok && col0 < a.N;  // the same in every epilogue thread
        if (e.issuer) {
            bulk_wait_read<1>();  // the copy issued from this box two chunks ago has read it
            if (EPI == Epi::kAdd && a.out_mode == 3) {
                if (active && !(e.rpending >> buf & 1))  // not prefetched
                    epi_load_resid<CONV>(e, tr, int(buf), col0, c1, c2, c3);
                e.rpending &= ~(1u << buf);
                // The next chunk's residual into the other box, once the previous chunk's store has read it: its
                // round trip overlaps this chunk.
                if (tile_ok && c + 32 < BN && col0 + 32 < a.N) {
                    bulk_wait_read<0>();
                    epi_load_resid<CONV>(e, tr, int(buf ^ 1), col0 + 32, c1, c2, c3);
                }
            }
        }
        named_barrier_sync<1, 128>();
        uint32_t acc[32];
        tmem_ld32(t_row + c, acc);
        tmem_wait_ld();
        if (active) {
            float b[32];
            load_bias32(sb, c, b);
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j)
                v[j] = __uint_as_float(acc[j]) + b[j];
            if constexpr (EPI == Epi::kResid) {
                if (row_ok) {
                    const int bsample = row / a.seg_rows;
                    const int within = row - bsample * a.seg_rows;
                    const float4* g4 = reinterpret_cast<const float4*>(
                        a.gate + long(bsample) * a.gate_bstride + (within < a.gate_split ? a.gate_alt_off : 0) + col0);
#pragma unroll
                    for (int j = 0; j < 8; ++j) {
                        float4 g = __ldg(g4 + j);
                        if (a.tanh_gate) {
                            g.x = tanh_fast(g.x);
                            g.y = tanh_fast(g.y);
                            g.z = tanh_fast(g.z);
                            g.w = tanh_fast(g.w);
                        }
                        v[4 * j] *= g.x;
                        v[4 * j + 1] *= g.y;
                        v[4 * j + 2] *= g.z;
                        v[4 * j + 3] *= g.w;
                    }
                }
            }
            if (EPI == Epi::kAdd && a.addvec && row_ok) {
                const float4* av =
                    reinterpret_cast<const float4*>(a.addvec + long(row / a.seg_rows) * a.addvec_stride + col0);
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 t = __ldg(av + j);
                    v[4 * j] += t.x;
                    v[4 * j + 1] += t.y;
                    v[4 * j + 2] += t.z;
                    v[4 * j + 3] += t.w;
                }
            }
            if (EPI == Epi::kAdd && a.out_mode == 3) {
                // On a timed-out wait the box is added as it is; the status bit reports the failure.
                mbar_wait(&e.rbar[buf], (e.rphase >> buf) & 1, status, kErrWaitEpiLoad, abort);
                e.rphase ^= 1u << buf;
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    const float4 t = *box_chunk(box, r, j);
                    v[4 * j] += t.x;
                    v[4 * j + 1] += t.y;
                    v[4 * j + 2] += t.z;
                    v[4 * j + 3] += t.w;
                }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
                *box_chunk(box, r, j) = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
            fence_proxy_async_smem();
            if constexpr (EPI == Epi::kAdd && CONV) {
                if (a.gn_part) {  // c1, c2, c3 = x0, y0, image of the pixel tile
                    const int chunk = ((c2 / a.conv_th) * (a.conv_wo / a.conv_tw) + c1 / a.conv_tw) * 4 + (r >> 5);
                    if (a.gn_cpg == 4)
                        gn_warp_stats<4>(a, v, row_ok, col0, c3, chunk);
                    else if (a.gn_cpg == 8)
                        gn_warp_stats<8>(a, v, row_ok, col0, c3, chunk);
                    else
                        gn_warp_stats<16>(a, v, row_ok, col0, c3, chunk);
                }
            }
        }
        named_barrier_sync<1, 128>();
        if (e.issuer && active) {
            if (a.out_mode == 2) {
                if constexpr (CONV)
                    tma_reduce_add_4d(to, box, col0, c1, c2, c3);
                else
                    tma_reduce_add_2d(to, box, col0, c1);
            } else {
                if constexpr (CONV)
                    tma_store_4d(to, box, col0, c1, c2, c3);
                else
                    tma_store_2d(to, box, col0, c1);
            }
            bulk_commit();
        }
    }
}

// Problem and problem-local tile of a global tile index (problem 0's tiles first).
__device__ __forceinline__ int gemm_problem(const GemmParams& P, int tile, int& local)
{
    const int p = (P.nprob > 1 && tile >= P.tiles0) ? 1 : 0;
    local = p ? tile - P.tiles0 : tile;
    return p;
}

template <int BN, Epi EPI, bool CONV>
__global__ void __launch_bounds__(kThreads, 1) k_gemm(const __grid_constant__ GemmParams P)
{
    using C = Cfg<BN, epi_staging(EPI)>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + C::kStages * C::kStageBytes;
    float* sbias = reinterpret_cast<float*>(staging + 2 * kEpiBox);  // [256] (add epilogue)
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::kStaging);
    uint64_t* empty = full + C::kStages;
    uint64_t* acc_full = empty + C::kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint64_t* rbar = drain + 1;  // [2] residual boxes of the TMA epilogue
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    int num_tiles = P.tiles0;
    if (P.nprob > 1)
        num_tiles += gemm_num_m(P.a[1], CONV) * ((P.a[1].N + BN - 1) / BN);
    uint32_t* status = P.a[0].status;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 128);
            mbar_init(&rbar[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        for (int p = 0; p < P.nprob; ++p) {
            prefetch_tmap(&P.ta[p]);
            prefetch_tmap(&P.tb[p]);
        }
    }
    grid_dep_wait();  // before TMEM allocation and the first global access
    if (warp == 1) {
        tmem_alloc(tmem_slot, C::kTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
                int local;
                const int p = gemm_problem(P, tile, local);
                const GemmArgs& args = P.a[p];
                const int num_m = gemm_num_m(args, CONV), num_n = (args.N + BN - 1) / BN;
                const int num_k = (args.K + kBK - 1) / kBK;
                int mb, nb;
                tile_coords(local, num_m, num_n, mb, nb);
                ConvWalk cw;
                if constexpr (CONV)
                    cw.start(args, mb);
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, status, kErrWaitEmpty, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + s * C::kStageBytes;
                    mbar_arrive_expect_tx(&full[s], C::kStageBytes);
                    if (P.test_stall && it == 0 && blockIdx.x == 0)
                        continue;  // the stage's bytes never arrive: full[0] cannot complete (failure-path test)
                    if constexpr (CONV) {
                        tma_load_4d(sa, &P.ta[p], &full[s], cw.c0, cw.x, cw.y, cw.b);
                        cw.next(args);
                    } else {
                        tma_load_2d(sa, &P.ta[p], &full[s], kb * kBK, mb * kBM);
                    }
                    tma_load_2d(sa + C::kABytes, &P.tb[p], &full[s], kb * kBK, nb * BN);
                }
            }
            if (!ok) {  // let the loads already issued land before the CTA can exit
                const uint32_t first = it > uint32_t(C::kStages) ? it - C::kStages : 0;
                for (uint32_t j = first; j < it; ++j)
                    mbar_wait(&full[j % C::kStages], (j / C::kStages) & 1, status, kErrWaitDrain, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = idesc_bf16_f32(kBM, BN);
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x, ++lt) {
                int local;
                const int p = gemm_problem(P, tile, local);
                const int num_k = (P.a[p].K + kBK - 1) / kBK;
                const uint32_t acc = lt & 1, acc_ph = (lt >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, status, kErrWaitAccEmpty, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&full[s], ph, status, kErrWaitFull, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
                    const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        mma_bf16_ss(d_tmem, desc_kmajor_sw128(a_addr + k * 32), desc_kmajor_sw128(b_addr + k * 32),
                                    idesc, (kb | k) != 0);
                    mma_commit(&empty[s]);
                }
                if (ok)
                    mma_commit(&acc_full[acc]);
            }
            // Every MMA must be complete before tensor memory is released.
            mma_commit(drain);
            mbar_wait(drain, 0, status, kErrWaitDrain, nullptr);
        }
    } else {
        const int q = warp & 3;  // the TMEM lane quarter this warp may access
        // kAdd and kResid always stage the bias; kBF16 only for tiles that leave through TMA (out_mode 4).
        constexpr bool kStageAlways = EPI == Epi::kAdd || EPI == Epi::kResid;
        const int et_idx = int(threadIdx.x) - 64;
        BiasStage<BN> bias_next;
        uint32_t lt = 0;
        EpiTma et;
        et.boxes = staging;
        et.rbar = rbar;
        et.issuer = threadIdx.x == 64;
        for (int tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++lt) {
            int local;
            const int p = gemm_problem(P, tile, local);
            const GemmArgs& args = P.a[p];
            const int num_m = gemm_num_m(args, CONV), num_n = (args.N + BN - 1) / BN;
            int mb, nb;
            tile_coords(local, num_m, num_n, mb, nb);
            const uint32_t acc = lt & 1, acc_ph = (lt >> 1) & 1;
            const float* sb = sbias;
            const bool stage = epi_tma(EPI) && (kStageAlways || args.out_mode);
            if (stage && lt == 0) {
                bias_next.load(args, nb * BN, et_idx);
                bias_next.store(sbias, et_idx);
            }
            if (EPI == Epi::kAdd && et.issuer && args.out_mode == 3) {  // first residual box, during the mainloop
                if constexpr (CONV) {
                    int pb, py0, px0;
                    conv_tile(args, mb, pb, py0, px0);
                    epi_prefetch_tile<true>(et, args, &P.tr[p], nb * BN, pb < args.conv_b, px0, py0, pb);
                } else {
                    const int prow0 = mb * kBM;
                    epi_prefetch_tile<false>(et, args, &P.tr[p], nb * BN, prow0 < args.M, prow0, 0, 0);
                }
            }
            const bool got = mbar_wait(&acc_full[acc], acc_ph, status, kErrWaitAccFull, abort_flag);
            // The staged bias and the TMA boxes synchronise the 128 epilogue threads: they leave together or not
            // at all.
            if (stage ? named_barrier_or<1, 128>(!got) : !got)
                break;
            bool has_next = false;
            if (epi_tma(EPI) && tile + int(gridDim.x) < num_tiles) {  // the next tile's bias, in flight while this tile drains
                int local2, mb2, nb2;
                const GemmArgs& a2 = P.a[gemm_problem(P, tile + int(gridDim.x), local2)];
                has_next = kStageAlways || a2.out_mode;
                if (has_next) {
                    tile_coords(local2, gemm_num_m(a2, CONV), (a2.N + BN - 1) / BN, mb2, nb2);
                    bias_next.load(a2, nb2 * BN, et_idx);
                }
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
            const int r = q * 32 + lane;
            if constexpr (CONV) {
                int b, y0, x0;
                conv_tile(args, mb, b, y0, x0);
                const int y = y0 + r / args.conv_tw, x = x0 + r % args.conv_tw;
                const int row = (b * args.conv_ho + y) * args.conv_wo + x;
                const bool row_ok = b < args.conv_b && y < args.conv_ho;
                if (epi_tma(EPI) && args.out_mode)
                    epilogue_tma<BN, EPI, true>(args, &P.to[p], &P.tr[p], t_row, r, row, row_ok, b < args.conv_b,
                                           nb * BN, x0, y0, b, sb, et, status, abort_flag);
                else
                    epilogue<BN, EPI>(args, t_row, row, row_ok, nb * BN, sb, staging + q * kQkvStage);
            } else {
                const int row0 = mb * kBM, row = row0 + r;
                if (epi_tma(EPI) && args.out_mode)
                    epilogue_tma<BN, EPI, false>(args, &P.to[p], &P.tr[p], t_row, r, row, row < args.M, row0 < args.M,
                                            nb * BN, row0, 0, 0, sb, et, status, abort_flag);
                else
                    epilogue<BN, EPI>(args, t_row, row, row < args.M, nb * BN, sb, staging + q * kQkvStage);
            }
            if (has_next) {
                // The TMA boxes' last barrier already follows every read of the current copy; a per-thread tile
                // that read it needs one.
                if (!args.out_mode && kStageAlways)
                    named_barrier_sync<1, 128>();
                bias_next.store(sbias, et_idx);
            }
            tc_fence_before();
            mbar_arrive(&acc_empty[acc]);
        }
        if (et.issuer) {
            epi_drain_resid(et, status);  // residual loads of a tile left early
            bulk_wait_all();              // the last boxes' copies finish before the CTA (and its shared memory) goes
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, C::kTmemCols);
    }
}


// The same GEMM on CTA pairs (cta_group::2): a cluster of two CTAs owns each 256 x BN tile. Each CTA loads its 128
// rows of X and half of the tile's W rows; the pair leader issues 256 x BN x 16 MMAs that read both CTAs' shared
// memory and accumulate each CTA's 128 rows in its own tensor memory; both CTAs run the epilogue on their rows. Per
// SM this halves the W traffic through shared memory and L2 of the 1-CTA tile. In convolution mode a pair tile is
// two consecutive 128-pixel output tiles (CTA rank r takes tile 2 m + r); a CTA whose tile lies past the last one
// (odd count) loads zeros through out-of-range TMA coordinates and stores nothing.
template <int BN, Epi EPI, bool CONV>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1) k_gemm2(const __grid_constant__ GemmParams P)
{
    using C = Cfg2<BN, epi_staging(EPI)>;
    constexpr int kPM = 2 * kBM;  // rows per pair tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* staging = smem + C::kStages * C::kStageBytes;
    float* sbias = reinterpret_cast<float*>(staging + 2 * kEpiBox);  // [256] (add epilogue)
    uint64_t* full = reinterpret_cast<uint64_t*>(staging + C::kStaging);
    uint64_t* empty = full + C::kStages;
    uint64_t* acc_full = empty + C::kStages;
    uint64_t* acc_empty = acc_full + 2;
    uint64_t* drain = acc_empty + 2;
    uint64_t* rbar = drain + 1;  // [2] residual boxes of the TMA epilogue
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(rbar + 2);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = cluster_ctarank();
    const bool leader = rank == 0;
    const int pair = blockIdx.x / 2, npairs = gridDim.x / 2;
    auto num_m_of = [&](const GemmArgs& a) { return (gemm_num_m(a, CONV) + 1) / 2; };
    int num_tiles = P.tiles0;
    if (P.nprob > 1)
        num_tiles += num_m_of(P.a[1]) * ((P.a[1].N + BN - 1) / BN);
    uint32_t* status = P.a[0].status;

    if (threadIdx.x == 0) {
        for (int s = 0; s < C::kStages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&acc_full[i], 1);
            mbar_init(&acc_empty[i], 2 * 128);  // the epilogue threads of both CTAs (leader's barrier)
            mbar_init(&rbar[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        for (int p = 0; p < P.nprob; ++p) {
            prefetch_tmap(&P.ta[p]);
            prefetch_tmap(&P.tb[p]);
        }
    }
    grid_dep_wait();  // before TMEM allocation and the first global access
    if (warp == 1) {
        tmem_alloc_pair(tmem_slot, C::kTmemCols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int tile = pair; tile < num_tiles && ok; tile += npairs) {
                int local;
                const int p = gemm_problem(P, tile, local);
                const GemmArgs& args = P.a[p];
                const int num_n = (args.N + BN - 1) / BN, num_k = (args.K + kBK - 1) / kBK;
                int mb, nb;
                tile_coords(local, num_m_of(args), num_n, mb, nb);
                ConvWalk cw;
                if constexpr (CONV)
                    cw.start(args, 2 * mb + int(rank));
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&empty[s], ph ^ 1, status, kErrWaitEmpty, abort_flag)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + s * C::kStageBytes;
                    if (leader)
                        mbar_arrive_expect_tx(&full[s], 2 * C::kStageBytes);  // both CTAs' loads land on it
                    if constexpr (CONV) {
                        tma_load_4d_pair(sa, &P.ta[p], &full[s], cw.c0, cw.x, cw.y, cw.b);
                        cw.next(args);
                    } else {
                        tma_load_2d_pair(sa, &P.ta[p], &full[s], kb * kBK, mb * kPM + int(rank) * kBM);
                    }
                    tma_load_2d_pair(sa + C::kABytes, &P.tb[p], &full[s], kb * kBK, nb * BN + int(rank) * (BN / 2));
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr uint32_t idesc = idesc_bf16_f32(kPM, BN);
            uint32_t it = 0, lt = 0;
            bool ok = true;
            for (int tile = pair; tile < num_tiles && ok; tile += npairs, ++lt) {
                int local;
                const int p = gemm_problem(P, tile, local);
                const int num_k = (P.a[p].K + kBK - 1) / kBK;
                const uint32_t acc = lt & 1, acc_ph = (lt >> 1) & 1;
                if (!mbar_wait(&acc_empty[acc], acc_ph ^ 1, status, kErrWaitAccEmpty, abort_flag))
                    break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_k; ++kb, ++it) {
                    const int s = it % C::kStages;
                    const uint32_t ph = (it / C::kStages) & 1;
                    if (!mbar_wait(&full[s], ph, status, kErrWaitFull, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(smem + s * C::kStageBytes);
                    const uint32_t b_addr = a_addr + C::kABytes;
#pragma unroll
                    for (int k = 0; k < kBK / 16; ++k)
                        mma_bf16_ss_pair(d_tmem, desc_kmajor_sw128(a_addr + k * 32),
                                         desc_kmajor_sw128(b_addr + k * 32), idesc, (kb | k) != 0);
                    mma_commit_pair(&empty[s]);
                }
                if (ok)
                    mma_commit_pair(&acc_full[acc]);
            }
            mma_commit_pair(drain);
            mbar_wait(drain, 0, status, kErrWaitDrain, nullptr);
        }
    } else {
        const int q = warp & 3;
        const uint32_t acc_empty_leader0 = map_to_cta(smem_u32(&acc_empty[0]), 0);
        // kAdd and kResid always stage the bias; kBF16 only for tiles that leave through TMA (out_mode 4).
        constexpr bool kStageAlways = EPI == Epi::kAdd || EPI == Epi::kResid;
        const int et_idx = int(threadIdx.x) - 64;
        BiasStage<BN> bias_next;
        uint32_t lt = 0;
        EpiTma et;
        et.boxes = staging;
        et.rbar = rbar;
        et.issuer = threadIdx.x == 64;
        for (int tile = pair; tile < num_tiles; tile += npairs, ++lt) {
            int local;
            const int p = gemm_problem(P, tile, local);
            const GemmArgs& args = P.a[p];
            int mb, nb;
            tile_coords(local, num_m_of(args), (args.N + BN - 1) / BN, mb, nb);
            const uint32_t acc = lt & 1, acc_ph = (lt >> 1) & 1;
            const float* sb = sbias;
            const bool stage = epi_tma(EPI) && (kStageAlways || args.out_mode);
            if (stage && lt == 0) {
                bias_next.load(args, nb * BN, et_idx);
                bias_next.store(sbias, et_idx);
            }
            if (EPI == Epi::kAdd && et.issuer && args.out_mode == 3) {  // first residual box, during the mainloop
                if constexpr (CONV) {
                    int pb, py0, px0;
                    conv_tile(args, 2 * mb + int(rank), pb, py0, px0);
                    epi_prefetch_tile<true>(et, args, &P.tr[p], nb * BN, pb < args.conv_b, px0, py0, pb);
                } else {
                    const int prow0 = mb * kPM + int(rank) * kBM;
                    epi_prefetch_tile<false>(et, args, &P.tr[p], nb * BN, prow0 < args.M, prow0, 0, 0);
                }
            }
            const bool got = mbar_wait(&acc_full[acc], acc_ph, status, kErrWaitAccFull, abort_flag);
            // The staged bias and the TMA boxes synchronise the 128 epilogue threads: they leave together or not
            // at all.
            if (stage ? named_barrier_or<1, 128>(!got) : !got)
                break;
            bool has_next = false;
            if (epi_tma(EPI) && tile + npairs < num_tiles) {  // the next tile's bias, in flight while this tile drains
                int local2, mb2, nb2;
                const GemmArgs& a2 = P.a[gemm_problem(P, tile + npairs, local2)];
                has_next = kStageAlways || a2.out_mode;
                if (has_next) {
                    tile_coords(local2, num_m_of(a2), (a2.N + BN - 1) / BN, mb2, nb2);
                    bias_next.load(a2, nb2 * BN, et_idx);
                }
            }
            tc_fence_after();
            const uint32_t t_row = tmem_base + (uint32_t(q * 32) << 16) + acc * BN;
            const int r = q * 32 + lane;
            if constexpr (CONV) {
                int b, y0, x0;
                conv_tile(args, 2 * mb + int(rank), b, y0, x0);
                const int y = y0 + r / args.conv_tw, x = x0 + r % args.conv_tw;
                const int row = (b * args.conv_ho + y) * args.conv_wo + x;
                const bool row_ok = b < args.conv_b && y < args.conv_ho;
                if (epi_tma(EPI) && args.out_mode)
                    epilogue_tma<BN, EPI, true>(args, &P.to[p], &P.tr[p], t_row, r, row, row_ok, b < args.conv_b,
                                           nb * BN, x0, y0, b, sb, et, status, abort_flag);
                else
                    epilogue<BN, EPI>(args, t_row, row, row_ok, nb * BN, sb, staging + q * kQkvStage);
            } else {
                const int row0 = mb * kPM + int(rank) * kBM, row = row0 + r;
                if (epi_tma(EPI) && args.out_mode)
                    epilogue_tma<BN, EPI, false>(args, &P.to[p], &P.tr[p], t_row, r, row, row < args.M, row0 < args.M,
                                            nb * BN, row0, 0, 0, sb, et, status, abort_flag);
                else
                    epilogue<BN, EPI>(args, t_row, row, row < args.M, nb * BN, sb, staging + q * kQkvStage);
            }
            if (has_next) {
                // The TMA boxes' last barrier already follows every read of the current copy; a per-thread tile
                // that read it needs one.
                if (!args.out_mode && kStageAlways)
                    named_barrier_sync<1, 128>();
                bias_next.store(sbias, et_idx);
            }
            tc_fence_before();
            if (leader)
                mbar_arrive(&acc_empty[acc]);
            else
                mbar_arrive_cluster(acc_empty_leader0 + acc * 8);
        }
        if (et.issuer) {
            epi_drain_resid(et, status);  // residual loads of a tile left early
            bulk_wait_all();              // the last boxes' copies finish before the CTA (and its shared memory) goes
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync_all();  // the leader's MMAs read this CTA's shared memory until here
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, C::kTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn()
{
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

template <int BN, Epi EPI, bool CONV>
cudaError_t launch_c(const GemmOp& op, cudaStream_t st)
{
    constexpr int kSmem = Cfg<BN, epi_staging(EPI)>::kSmem;
    static std::atomic<uint64_t> attr_devs{0};
    const cudaError_t e = smem_limit_once(attr_devs, k_gemm<BN, EPI, CONV>, kSmem);
    if (e != cudaSuccess)
        return e;
    launch_k(k_gemm<BN, EPI, CONV>, op.grid, kThreads, kSmem, st, op.p);
    count_launch();
    return cudaGetLastError();
}

template <int BN, Epi EPI, bool CONV>
cudaError_t launch_pair(const GemmOp& op, cudaStream_t st)
{
    if constexpr (BN >= 128 && (BN / 2) % 16 == 0) {
        constexpr int kSmem = Cfg2<BN, epi_staging(EPI)>::kSmem;
        static std::atomic<uint64_t> attr_devs{0};
        const cudaError_t e = smem_limit_once(attr_devs, k_gemm2<BN, EPI, CONV>, kSmem);
        if (e != cudaSuccess)
            return e;
        launch_k(k_gemm2<BN, EPI, CONV>, op.grid, kThreads, kSmem, st, op.p);
        count_launch();
        return cudaGetLastError();
    }
    return cudaErrorInvalidValue;
}

template <int BN, Epi EPI>
cudaError_t launch_t(const GemmOp& op, cudaStream_t st)
{
    // Convolutions only use the epilogues a conv needs (plain, activation, add), which keeps the instantiations few.
    if constexpr (EPI == Epi::kBF16 || EPI == Epi::kAdd) {
        if (op.conv)
            return op.pair ? launch_pair<BN, EPI, true>(op, st) : launch_c<BN, EPI, true>(op, st);
    }
    if (op.pair)
        return launch_pair<BN, EPI, false>(op, st);
    return launch_c<BN, EPI, false>(op, st);
}

template <int BN>
cudaError_t launch_bn(const GemmOp& op, cudaStream_t st)
{
    switch (op.epi) {
    case Epi::kAdd: return launch_t<BN, Epi::kAdd>(op, st);
    case Epi::kHeads: return launch_t<BN, Epi::kHeads>(op, st);
    case Epi::kBF16: return launch_t<BN, Epi::kBF16>(op, st);
    case Epi::kF32: return launch_t<BN, Epi::kF32>(op, st);
    case Epi::kResid: return launch_t<BN, Epi::kResid>(op, st);
    case Epi::kQkv: return launch_t<BN, Epi::kQkv>(op, st);
    case Epi::kSwiGLU: return launch_t<BN, Epi::kSwiGLU>(op, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace

GemmTile gemm_pick_tile(long M, int N, bool allow_pairs, int only_bn)
{
    // Makespan in units of one 128-column mainloop: rounds of tiles over the SMs (pair tiles over pairs of SMs, each
    // SM doing 128 of the 256 rows), times the tile width, times a shared-memory factor. Per SM and MMA cycle a
    // 1-CTA tile reads 8192 / BN + 64 bytes of X and W operands, a pair tile 8192 / BN + 32; above ~88 B/clk the
    // tensor pipe waits for shared memory (calibrated on the FFN-up shape: 1-CTA 256 1.10x and 192 1.22x slower
    // than the 256 pair).
    const long sms = num_sms();
    GemmTile best{0, false};
    double best_cost = 0;
    for (int pairs = 0; pairs <= (allow_pairs ? 1 : 0); ++pairs)
        for (int bn : {256, 192, 160, 128, 64}) {
            if (only_bn && bn != only_bn)
                continue;
            if (N % bn && !(bn == 64 && N % 32 == 0))
                continue;
            if (pairs && bn < 128)
                continue;
            const long rows = pairs ? 2 * kBM : kBM, slots = pairs ? sms / 2 : sms;
            const long tiles = ((M + rows - 1) / rows) * ((N + bn - 1) / bn);
            const double bpc = 8192.0 / bn + (pairs ? 32.0 : 64.0);
            const double cost = double((tiles + slots - 1) / slots) * bn * std::max(1.0, bpc / 88.0);
            if (!best.bn || cost < best_cost - 1e-9) {
                best = GemmTile{bn, pairs != 0};
                best_cost = cost;
            }
        }
    return best;
}

int gemm_pick_bn(long M, int N, bool pairs) { return gemm_pick_tile(M, N, pairs).bn; }

int num_sms()
{
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0)
            n = 148;
    }
    return n;
}

bool make_tmap_bf16_2d(CUtensorMap* m, const void* ptr, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                       uint32_t box_inner, uint32_t box_outer, const char** err)
{
    auto fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (row_bytes & 15)) {
        *err = "tensor map: base or row stride not 16-byte aligned";
        return false;
    }
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) {
        *err = "cuTensorMapEncodeTiled failed";
        return false;
    }
    return true;
}

namespace {

bool tma_epilogue_enabled()
{
    static const bool on = [] {
        const char* v = std::getenv("MKB_TMA_EPI");
        return !(v && v[0] == '0');
    }();
    return on;
}

bool make_tmap_f32(CUtensorMap* m, const void* ptr, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
                   const cuuint32_t* box, const char** err)
{
    auto fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    const cuuint32_t es[4] = {1, 1, 1, 1};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, cuuint32_t(rank), const_cast<void*>(ptr), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        *err = "gemm: output tensor map encoding failed";
        return false;
    }
    return true;
}

// Chooses how a kAdd problem with fp32 output leaves the SM (GemmArgs::out_mode) and encodes its output and
// residual boxes: 32 columns x the tile's 128 rows, or for a convolution 32 channels x tw x th pixels of one image
// over the output viewed as [B][Ho][Wo][N]. Outputs TMA cannot address (unaligned) keep the per-thread stores.
bool prepare_out_boxes(GemmParams& P, int prob, Epi epi, int bn, bool conv, const char** err)
{
    GemmArgs& a = P.a[prob];
    a.out_mode = 0;
    if (epi == Epi::kResid) {  // the gated residual, always in place: reduce-add into resid
        if (!tma_epilogue_enabled() || (reinterpret_cast<uintptr_t>(a.resid) & 15) || (a.ldr & 3) || conv)
            return true;
        const cuuint64_t dims[2] = {cuuint64_t(a.N), cuuint64_t(a.M)};
        const cuuint64_t strides[1] = {cuuint64_t(a.ldr) * 4};
        const cuuint32_t box[2] = {32, cuuint32_t(kBM)};
        if (!make_tmap_f32(&P.to[prob], a.resid, 2, dims, strides, box, err))
            return false;
        a.out_mode = 2;
        return true;
    }
    if (epi == Epi::kBF16) {  // bf16 output: 64-column boxes, tile widths that are multiples of 64
        if (!tma_epilogue_enabled() || conv || bn % 64 || !a.out || (reinterpret_cast<uintptr_t>(a.out) & 15) ||
            (a.ldo & 7))
            return true;
        const cuuint64_t dims[2] = {cuuint64_t(a.N), cuuint64_t(a.M)};
        const cuuint64_t strides[1] = {cuuint64_t(a.ldo) * 2};
        const cuuint32_t box[2] = {64, cuuint32_t(kBM)};
        auto fn = encode_fn();
        const cuuint32_t es[2] = {1, 1};
        if (!fn || fn(&P.to[prob], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, a.out, dims, strides, box, es,
                      CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
            *err = "gemm: output tensor map encoding failed";
            return false;
        }
        a.out_mode = 4;
        return true;
    }
    if (!tma_epilogue_enabled() || !a.out_f32 || !a.out)
        return true;
    if ((reinterpret_cast<uintptr_t>(a.out) & 15) || (a.ldo & 3) ||
        (a.add_resid && ((reinterpret_cast<uintptr_t>(a.add_resid) & 15) || (a.ld_add_resid & 3))))
        return true;
    const int mode = !a.add_resid ? 1 : (a.add_resid == a.out && a.ld_add_resid == a.ldo) ? 2 : 3;
    auto encode = [&](CUtensorMap* m, const void* ptr, long ld) {
        const cuuint64_t row_bytes = cuuint64_t(ld) * 4;
        if (conv) {
            const cuuint64_t dims[4] = {cuuint64_t(a.N), cuuint64_t(a.conv_wo), cuuint64_t(a.conv_ho),
                                        cuuint64_t(a.conv_b)};
            const cuuint64_t strides[3] = {row_bytes, row_bytes * a.conv_wo, row_bytes * a.conv_wo * a.conv_ho};
            const cuuint32_t box[4] = {32, cuuint32_t(a.conv_tw), cuuint32_t(a.conv_th), 1};
            return make_tmap_f32(m, ptr, 4, dims, strides, box, err);
        }
        const cuuint64_t dims[2] = {cuuint64_t(a.N), cuuint64_t(a.M)};
        const cuuint64_t strides[1] = {row_bytes};
        const cuuint32_t box[2] = {32, cuuint32_t(kBM)};
        return make_tmap_f32(m, ptr, 2, dims, strides, box, err);
    };
    if (!encode(&P.to[prob], a.out, a.ldo))
        return false;
    if (mode == 3 && !encode(&P.tr[prob], a.add_resid, a.ld_add_resid))
        return false;
    a.out_mode = mode;
    return true;
}

// Checks of the epilogue arguments shared by the GEMM and the convolution.
bool check_epilogue(Epi epi, const GemmArgs& args, int bn, const char** err)
{
    if (bn != 64 && bn != 128 && bn != 160 && bn != 192 && bn != 256) {
        *err = "gemm: tile width must be 64, 128, 160, 192 or 256";
        return false;
    }
    if (epi == Epi::kQkv && (bn < 128 || args.D % bn || args.N != 3 * args.D || !args.qh || !args.kh || !args.vh)) {
        *err = "gemm: qkv epilogue needs N = 3 D, D a multiple of the tile width, and q/k/v outputs";
        return false;
    }
    if (epi == Epi::kQkv && args.head_group > 0 &&
        ((args.D / 128) % args.head_group || args.group_chunk <= 0 || !args.group_dst)) {
        *err = "gemm: qkv head groups must divide the heads and have a positive chunk and a destination table";
        return false;
    }
    if (epi == Epi::kSwiGLU && (bn != 256 || args.N % bn)) {
        *err = "gemm: swiglu epilogue needs 256-wide tiles (128 gate + 128 up columns) and N a multiple of 256";
        return false;
    }
    if (epi == Epi::kResid && (!args.resid || !args.gate || (args.ldr & 3))) {
        *err = "gemm: residual epilogue needs resid, gate, and ldr a multiple of 4";
        return false;
    }
    if ((epi == Epi::kBF16 || epi == Epi::kSwiGLU) && (!args.out || (args.ldo & 7))) {
        *err = "gemm: bf16 output needs out and ldo a multiple of 8";
        return false;
    }
    if (epi == Epi::kF32 && (!args.out || (args.ldo & 3))) {
        *err = "gemm: f32 output needs out and ldo a multiple of 4";
        return false;
    }
    if (epi == Epi::kAdd && (!args.out || (args.ldo & (args.out_f32 ? 3 : 7)) || (args.add_resid && (args.ld_add_resid & 3)))) {
        *err = "gemm: add epilogue needs out with an aligned ldo (and an aligned residual)";
        return false;
    }
    if (epi == Epi::kHeads && ((args.head_dim != 64 && args.head_dim != 128) || args.D % args.head_dim ||
                               args.part0 < 0 || (args.N + args.D - 1) / args.D + args.part0 > 3)) {
        *err = "gemm: heads epilogue needs head_dim 64 or 128 dividing D and at most 3 parts";
        return false;
    }
    return true;
}

}  // namespace

bool gemm_prepare(GemmOp& op, Epi epi, const void* X, long ldx, const void* W, long ldw, const GemmArgs& args,
                  int bn, const char** err)
{
    op.ready = false;
    op.conv = false;
    op.p.nprob = 1;
    if (args.M <= 0 || args.N <= 0 || args.K <= 0 || args.N % 32 || args.K % 8) {
        *err = "gemm: M, N, K must be positive, N a multiple of 32, K a multiple of 8";
        return false;
    }
    if (!check_epilogue(epi, args, bn, err))
        return false;
    if (!make_tmap_bf16_2d(&op.p.ta[0], X, uint64_t(args.K), uint64_t(args.M), uint64_t(ldx) * 2, kBK, kBM, err))
        return false;
    if (!make_tmap_bf16_2d(&op.p.tb[0], W, uint64_t(args.K), uint64_t(args.N), uint64_t(ldw) * 2, kBK, uint32_t(bn),
                           err))
        return false;
    op.p.a[0] = args;
    if (epi_tma(epi) && !prepare_out_boxes(op.p, 0, epi, bn, false, err))
        return false;
    op.p.nprob = 1;
    op.pair = false;
    op.w_ptr[0] = W;
    op.ldw[0] = ldw;
    op.p.tiles0 = ((args.M + kBM - 1) / kBM) * ((args.N + bn - 1) / bn);
    op.epi = epi;
    op.bn = bn;
    op.grid = op.p.tiles0 < num_sms() ? op.p.tiles0 : num_sms();
    op.ready = true;
    return true;
}

bool gemm_add_problem(GemmOp& op, const void* X, long ldx, const void* W, long ldw, const GemmArgs& args,
                      const char** err)
{
    if (!op.ready || op.conv || op.pair || op.p.nprob != 1) {
        *err = "gemm: a second problem needs a prepared single 1-CTA GEMM";
        return false;
    }
    if (args.M <= 0 || args.N <= 0 || args.K <= 0 || args.N % 32 || args.K % 8) {
        *err = "gemm: M, N, K must be positive, N a multiple of 32, K a multiple of 8";
        return false;
    }
    if (!check_epilogue(op.epi, args, op.bn, err))
        return false;
    if (!make_tmap_bf16_2d(&op.p.ta[1], X, uint64_t(args.K), uint64_t(args.M), uint64_t(ldx) * 2, kBK, kBM, err))
        return false;
    if (!make_tmap_bf16_2d(&op.p.tb[1], W, uint64_t(args.K), uint64_t(args.N), uint64_t(ldw) * 2, kBK,
                           uint32_t(op.bn), err))
        return false;
    op.p.a[1] = args;
    op.p.a[1].status = op.p.a[0].status;
    if (epi_tma(op.epi) && !prepare_out_boxes(op.p, 1, op.epi, op.bn, false, err))
        return false;
    op.p.nprob = 2;
    op.w_ptr[1] = W;
    op.ldw[1] = ldw;
    const int tiles = op.p.tiles0 + ((args.M + kBM - 1) / kBM) * ((args.N + op.bn - 1) / op.bn);
    op.grid = tiles < num_sms() ? tiles : num_sms();
    return true;
}

int conv_tile_w(int Wo)
{
    int tw = 128;
    while (tw > 1 && Wo % tw)
        tw >>= 1;
    return tw;
}

int conv_gn_chunks(int Ho, int Wo)
{
    const int tw = conv_tile_w(Wo), th = 128 / tw;
    return (Wo / tw) * ((Ho + th - 1) / th) * 4;
}

bool conv_prepare(GemmOp& op, Epi epi, const void* X, int B, int Hi, int Wi, int C, const void* W, int Cout,
                  int taps, int stride, const GemmArgs& args_in, int bn, const char** err)
{
    op.ready = false;
    if (epi != Epi::kBF16 && epi != Epi::kAdd) {
        *err = "conv: only the plain / activation and add epilogues";
        return false;
    }
    if ((taps != 9 && taps != 1) || (stride != 1 && stride != 2) || (taps == 1 && stride != 1) || B <= 0 ||
        Hi <= 0 || Wi <= 0 || C <= 0 || C % kBK || Cout <= 0 || Cout % 32) {
        *err = "conv: taps 9 (3x3, padding 1) or 1, stride 1 or 2 (3x3 only), C a multiple of 64, Cout of 32";
        return false;
    }
    GemmArgs a = args_in;
    const int Ho = taps == 9 ? (Hi + 2 - 3) / stride + 1 : Hi, Wo = taps == 9 ? (Wi + 2 - 3) / stride + 1 : Wi;
    // Tile: tw columns x (128 / tw) rows of output pixels, tw the widest power of two <= 128 dividing Wo.
    const int tw = conv_tile_w(Wo);
    if (tw < 8) {
        *err = "conv: the output width must be a multiple of 8";
        return false;
    }
    a.conv_b = B;
    a.conv_hi = Hi;
    a.conv_wi = Wi;
    a.conv_c = C;
    a.conv_ho = Ho;
    a.conv_wo = Wo;
    a.conv_stride = stride;
    a.conv_taps = taps;
    a.conv_pad = taps == 9 ? 1 : 0;
    a.conv_tw = tw;
    a.conv_th = 128 / tw;
    a.M = B * Ho * Wo;
    a.N = Cout;
    a.K = taps * C;
    if (a.seg_rows == (1 << 30))
        a.seg_rows = Ho * Wo;  // per-sample vectors index by image
    if (a.gn_part) {
        if (epi != Epi::kAdd || !a.out_f32 || (a.gn_cpg != 4 && a.gn_cpg != 8 && a.gn_cpg != 16) ||
            (reinterpret_cast<uintptr_t>(a.gn_part) & 15)) {
            *err = "conv: GroupNorm statistics need the fp32 add epilogue, 4, 8 or 16 channels a group, 16-byte "
                   "aligned partials";
            return false;
        }
        a.gn_chunks = conv_gn_chunks(Ho, Wo);
    }
    if (!check_epilogue(epi, a, bn, err))
        return false;
    auto fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    if (reinterpret_cast<uintptr_t>(X) & 15) {
        *err = "conv: input not 16-byte aligned";
        return false;
    }
    // Input [B][Hi][Wi][C] read as windows of 64 channels x (tw * stride) x (th * stride) pixels, every stride-th
    // pixel, 128-byte swizzle: the smem tile is 128 rows (pixels) of 64 channels like the GEMM's A tile.
    cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(Wi), cuuint64_t(Hi), cuuint64_t(B)};
    cuuint64_t strides[3] = {cuuint64_t(C) * 2, cuuint64_t(Wi) * C * 2, cuuint64_t(Hi) * Wi * C * 2};
    cuuint32_t box[4] = {cuuint32_t(kBK), cuuint32_t(tw * stride), cuuint32_t((128 / tw) * stride), 1};
    cuuint32_t es[4] = {1, cuuint32_t(stride), cuuint32_t(stride), 1};
    if (box[1] > 256 || box[2] > 256) {
        *err = "conv: tile window too large";
        return false;
    }
    if (fn(&op.p.ta[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(X), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        *err = "conv: input tensor map encoding failed";
        return false;
    }
    if (!make_tmap_bf16_2d(&op.p.tb[0], W, uint64_t(a.K), uint64_t(Cout), uint64_t(a.K) * 2, kBK, uint32_t(bn), err))
        return false;
    op.p.a[0] = a;
    if (epi_tma(epi) && !prepare_out_boxes(op.p, 0, epi, bn, true, err))
        return false;
    if (a.gn_part && !op.p.a[0].out_mode) {
        *err = "conv: GroupNorm statistics need the output boxes of the TMA epilogue";
        return false;
    }
    op.p.nprob = 1;
    op.epi = epi;
    op.bn = bn;
    op.conv = true;
    op.pair = false;
    op.w_ptr[0] = W;
    op.ldw[0] = a.K;
    const int tiles = B * (Wo / tw) * ((Ho + a.conv_th - 1) / a.conv_th) * ((Cout + bn - 1) / bn);
    op.p.tiles0 = tiles;
    op.grid = tiles < num_sms() ? tiles : num_sms();
    op.ready = true;
    return true;
}

bool gemm_use_pairs(GemmOp& op, const char** err)
{
    if (!op.ready || op.bn < 128 || (op.conv && op.p.nprob != 1)) {
        *err = "gemm: CTA pairs need a prepared GEMM or convolution with tile width >= 128";
        return false;
    }
    int tiles = 0;
    for (int p = 0; p < op.p.nprob; ++p) {
        const GemmArgs& a = op.p.a[p];
        // W tiles are loaded half per CTA: re-encode W's map with a box of bn / 2 rows.
        CUtensorMap m;
        if (!make_tmap_bf16_2d(&m, op.w_ptr[p], uint64_t(a.K), uint64_t(a.N), uint64_t(op.ldw[p]) * 2, kBK,
                               uint32_t(op.bn / 2), err))
            return false;
        op.p.tb[p] = m;
        // Pair tiles: 256 rows, or two consecutive 128-pixel output tiles of a convolution.
        const int m128 = op.conv ? a.conv_b * (a.conv_wo / a.conv_tw) * ((a.conv_ho + a.conv_th - 1) / a.conv_th)
                                 : (a.M + kBM - 1) / kBM;
        const int t = ((m128 + 1) / 2) * ((a.N + op.bn - 1) / op.bn);
        if (p == 0)
            op.p.tiles0 = t;
        tiles += t;
    }
    const int pairs = num_sms() / 2;
    op.grid = 2 * (tiles < pairs ? tiles : pairs);
    op.pair = true;
    return true;
}

cudaError_t gemm_launch(const GemmOp& op, cudaStream_t st)
{
    if (!op.ready)
        return cudaErrorInvalidValue;
    switch (op.bn) {
    case 64: return launch_bn<64>(op, st);
    case 128: return launch_bn<128>(op, st);
    case 160: return launch_bn<160>(op, st);
    case 192: return launch_bn<192>(op, st);
    case 256: return launch_bn<256>(op, st);
    }
    return cudaErrorInvalidValue;
}

}  // namespace mkb
