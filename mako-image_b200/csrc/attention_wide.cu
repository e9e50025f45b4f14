// Single-head flash attention at head dim 256 or 512 on tcgen05: the VAE decoder's mid-block attention
// (Engine::vae_attention, src/image/engine.cpp:748-778: softmax(q k^T / sqrt(C)) v over every pixel of the latent
// image, C = 512 channels), which the reference runs as a score GEMM, a row softmax and a P V GEMM.
//
// At d = 512 one query tile's output (128 x 512 fp32) fills all of tensor memory, so each 128-query tile is split
// over two CTAs by output columns: CTA (tile, half) computes O[:, half * d/2 .. + d/2]. Both compute the full scores
// (the contraction runs over all d), which costs a third more MMA work than one pass but keeps every tile's scores,
// P and its O half in one SM's tensor memory: S_even [0, 128), S_odd [128, 256), O [256, 256 + d/2).
//   warp 0     TMA: the Q tile once (d/64 panels of 128 x 64, resident), then K panels (d/64 per key tile) and the
//              CTA's V panels (d/128 per key tile) through one ring of 16 KB stages, in the order the MMA warp
//              consumes them: K_0, K_1, V_0, K_2, V_1, K_3, ...
//   warp 1     MMA: S_j = Q K_j^T into S_{j&1}; after the softmax has published P_j, O += P_j V_j (P from tensor
//              memory), then S_{j+2}. The scores of the next key tile are computed while the softmax works on these.
//   warps 2-3  idle
//   warps 4-7  softmax, one thread per query row: running max with lazy rescaling (O is rescaled only when a row's
//              max grows by more than 2^8, after the previous P V has landed), P = 2^(S - m) as bf16 over the first
//              64 columns of S, and at the end O / l as bf16 into the output rows.
// Every wait is bounded (sm100.cuh); a wait that runs out sets kErrAttnWait and the CTA leaves.
#include "attention.cuh"
#include "common.cuh"
#include "launch.cuh"
#include "sm100.cuh"

#include <cudaTypedefs.h>
#include <atomic>
#include <cmath>
#include <mutex>

namespace mkb {

namespace {

constexpr int kWThreads = 256;
constexpr int kWTile = 128;                  // query rows per CTA, keys per key tile
constexpr int kWPanel = kWTile * 64 * 2;     // 128 rows x 64 bf16 with the 128-byte swizzle: 16 KB
constexpr uint32_t kWTmemCols = 512;
constexpr float kWRescale = 8.0f;            // log2 units
// K / V panels in flight: as many as fit beside the resident Q tile in 227 KB.
template <int D>
constexpr int kWStages = D == 512 ? 6 : 8;
template <int D>
constexpr int kWSmem = 1024 + (D / 64) * kWPanel + kWStages<D> * kWPanel + 256;
static_assert(kWSmem<512> <= 227 * 1024 && kWSmem<256> <= 227 * 1024, "shared memory over the per-CTA limit");

__device__ __forceinline__ float wex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

template <int D>
__global__ void __launch_bounds__(kWThreads, 1) k_attn_wide(const __grid_constant__ CUtensorMap tm, const AttnWideArgs a)
{
    constexpr int NQ = D / 64;   // Q / K panels: the contraction in 64-wide steps
    constexpr int NV = D / 128;  // V panels of this CTA's output half
    constexpr int DH = D / 2;
    constexpr int kWS = kWStages<D>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* sQ = smem;
    uint8_t* ring = smem + NQ * kWPanel;
    uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kWS * kWPanel);
    uint64_t* q_full = bars;
    uint64_t* full = bars + 1;            // [kWS]
    uint64_t* empty = full + kWS;         // [kWS]
    uint64_t* s_full = empty + kWS;       // [2] by key-tile parity
    uint64_t* p_full = s_full + 2;            // [2]
    uint64_t* o_done = p_full + 2;            // [2]
    uint64_t* drain = o_done + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = blockIdx.x * kWTile, half = blockIdx.y;
    const int nkv = (a.n + kWTile - 1) / kWTile;

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < kWS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[i], 128);
            mbar_init(&o_done[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0)
        prefetch_tmap(&tm);
    grid_dep_wait();
    if (warp == 1) {
        tmem_alloc(tmem_slot, kWTmemCols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            mbar_arrive_expect_tx(q_full, NQ * kWPanel);
            for (int c = 0; c < NQ; ++c)
                tma_load_2d(sQ + c * kWPanel, &tm, q_full, a.q_col + 64 * c, q0);
            auto put = [&](int col, int row) {
                const uint32_t s = it % kWS, ph = (it / kWS) & 1;
                if (!mbar_wait(&empty[s], ph ^ 1, a.status, kErrAttnWait, abort_flag))
                    return false;
                mbar_arrive_expect_tx(&full[s], kWPanel);
                tma_load_2d(ring + s * kWPanel, &tm, &full[s], col, row);
                ++it;
                return true;
            };
            auto put_k = [&](int j) {
                for (int c = 0; c < NQ && ok; ++c)
                    ok = put(a.k_col + 64 * c, j * kWTile);
            };
            auto put_v = [&](int j) {
                for (int p = 0; p < NV && ok; ++p)
                    ok = put(a.v_col + half * DH + 64 * p, j * kWTile);
            };
            put_k(0);
            if (nkv > 1)
                put_k(1);
            for (int j = 0; j < nkv && ok; ++j) {
                put_v(j);
                if (j + 2 < nkv)
                    put_k(j + 2);
            }
            if (!ok) {  // let the loads already issued land before the CTA can exit
                mbar_wait(q_full, 0, a.status, kErrWaitDrain, nullptr);
                for (uint32_t j = it > uint32_t(kWS) ? it - kWS : 0; j < it; ++j)
                    mbar_wait(&full[j % kWS], (j / kWS) & 1, a.status, kErrWaitDrain, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, 0, 0);
            constexpr uint32_t idesc_o = idesc_bf16_f32(128, 64, 0, 1);  // V is MN-major (its columns contiguous)
            const uint32_t q_addr = smem_u32(sQ);
            uint32_t it = 0;
            bool ok = mbar_wait(q_full, 0, a.status, kErrAttnWait, abort_flag);
            auto take = [&](uint32_t& addr) {
                const uint32_t s = it % kWS, ph = (it / kWS) & 1;
                if (!mbar_wait(&full[s], ph, a.status, kErrAttnWait, abort_flag))
                    return false;
                tc_fence_after();
                addr = smem_u32(ring + s * kWPanel);
                return true;
            };
            auto give = [&] {  // the stage is free once the MMAs issued on it have read it
                mma_commit(&empty[it % kWS]);
                ++it;
            };
            auto issue_s = [&](int j) {
                const uint32_t d = tmem + (j & 1) * 128;
                for (int c = 0; c < NQ && ok; ++c) {
                    uint32_t k_addr;
                    if (!(ok = take(k_addr)))
                        break;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
                        mma_bf16_ss(d, desc_kmajor_sw128(q_addr + c * kWPanel + kk * 32),
                                    desc_kmajor_sw128(k_addr + kk * 32), idesc_s, (c > 0) || (kk > 0));
                    give();
                }
                if (ok)
                    mma_commit(&s_full[j & 1]);
            };
            auto issue_pv = [&](int j) {
                if (!(ok = mbar_wait(&p_full[j & 1], (j >> 1) & 1, a.status, kErrAttnWait, abort_flag)))
                    return;
                tc_fence_after();
                const uint32_t p_col = tmem + (j & 1) * 128;
                for (int p = 0; p < NV && ok; ++p) {
                    uint32_t v_addr;
                    if (!(ok = take(v_addr)))
                        break;
#pragma unroll
                    for (int k = 0; k < 8; ++k)  // 16 keys a step: P columns 8k.., V rows 16k..
                        mma_bf16_ts(tmem + 256 + 64 * p, p_col + 8 * k,
                                    desc_mnmajor_sw128(v_addr + k * 2048, kWPanel, 1024), idesc_o, (j > 0) || (k > 0));
                    give();
                }
                if (ok)
                    mma_commit(&o_done[j & 1]);
            };
            if (ok) {
                issue_s(0);
                if (nkv > 1 && ok)
                    issue_s(1);
                for (int j = 0; j < nkv && ok; ++j) {
                    issue_pv(j);
                    if (j + 2 < nkv && ok)
                        issue_s(j + 2);
                }
            }
            mma_commit(drain);  // arrives once every MMA issued above has completed
            mbar_wait(drain, 0, a.status, kErrWaitDrain, nullptr);
        }
    } else if (warp >= 4) {
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t t_lane = tmem + (uint32_t(quarter * 32) << 16);
        const float sc = a.scale_log2;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            const uint32_t col_s = (j & 1) * 128;
            if (!mbar_wait(&s_full[j & 1], (j >> 1) & 1, a.status, kErrAttnWait, abort_flag)) {
                ok = false;
                break;
            }
            tc_fence_after();
            uint32_t s[128];
            tmem_ld32(t_lane + col_s, *reinterpret_cast<uint32_t(*)[32]>(&s[0]));
            tmem_ld32(t_lane + col_s + 32, *reinterpret_cast<uint32_t(*)[32]>(&s[32]));
            tmem_ld32(t_lane + col_s + 64, *reinterpret_cast<uint32_t(*)[32]>(&s[64]));
            tmem_ld32(t_lane + col_s + 96, *reinterpret_cast<uint32_t(*)[32]>(&s[96]));
            tmem_wait_ld();
            const int valid = min(kWTile, a.n - j * kWTile);  // keys past the end read as zeros: masked
            if (valid < kWTile) {
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    if (i >= valid)
                        s[i] = __float_as_uint(-INFINITY);
            }
            // Row max as 8 independent chains of 3-input max.
            float mc[8];
#pragma unroll
            for (int u = 0; u < 8; ++u)
                mc[u] = fmaxf(__uint_as_float(s[2 * u]), __uint_as_float(s[2 * u + 1]));
#pragma unroll
            for (int i = 16; i < 128; i += 16)
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    mc[u] = fmax3(mc[u], __uint_as_float(s[i + 2 * u]), __uint_as_float(s[i + 2 * u + 1]));
            float mx = fmax3(fmax3(mc[0], mc[1], mc[2]), fmax3(mc[3], mc[4], mc[5]), fmaxf(mc[6], mc[7]));
            mx *= sc;
            const bool need = mx > m_used + kWRescale;
            if (__any_sync(0xffffffffu, need)) {
                const float m_new = need ? mx : m_used;
                const float f = wex2(m_used - m_new);  // 0 on the first tile
                l *= f;
                if (j > 0) {  // O holds P V of tiles < j: rescale it once the last of them has landed
                    if (!mbar_wait(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.status, kErrAttnWait, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
#pragma unroll 1
                    for (int c = 0; c < DH / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(t_lane + 256 + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
                        uint32_t lo[16], hi[16];
#pragma unroll
                        for (int i = 0; i < 16; ++i) {
                            lo[i] = o[i];
                            hi[i] = o[16 + i];
                        }
                        tmem_st16(t_lane + 256 + c * 32, lo);
                        tmem_st16(t_lane + 256 + c * 32 + 16, hi);
                    }
                }
                m_used = m_new;
            }
            // x = s * scale - m two scores per packed FMA; every eighth pair's 2^x on the FMA pipe (a polynomial) to
            // offload the SFU; the row sum in 4 packed accumulators.
            const float2 sc2 = make_float2(sc, sc), nm2 = make_float2(-m_used, -m_used);
            float2 ls[4] = {};
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                uint32_t p[16];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const int k = c * 32 + 2 * i;
                    const float2 x = ffma2(make_float2(__uint_as_float(s[k]), __uint_as_float(s[k + 1])), sc2, nm2);
                    float2 e;
                    if (i % 8 == 7) {
                        e = ex2_poly2(x);
                    } else {
                        e.x = wex2(x.x);
                        e.y = wex2(x.y);
                    }
                    ls[i & 3] = fadd2(ls[i & 3], e);
                    p[i] = pack_bf16x2(e.x, e.y);
                }
                tmem_st16(t_lane + col_s + c * 16, p);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(&p_full[j & 1]);
            const float2 l01 = fadd2(fadd2(ls[0], ls[1]), fadd2(ls[2], ls[3]));
            l += l01.x + l01.y;
        }
        const int jl = nkv - 1;
        if (ok && nkv > 0 && mbar_wait(&o_done[jl & 1], (jl >> 1) & 1, a.status, kErrAttnWait, abort_flag)) {
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const int row = q0 + r;
            __nv_bfloat16* dst = row < a.n ? a.out + long(row) * a.ldo + half * DH : nullptr;
#pragma unroll 1
            for (int c = 0; c < DH / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(t_lane + 256 + c * 32, o);
                tmem_wait_ld();
                if (dst) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        d4[i] = make_uint4(
                            pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                            pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                            pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                            pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, kWTmemCols);
    }
}

PFN_cuTensorMapEncodeTiled_v12000 wide_encode_fn()
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

template <int D>
cudaError_t wide_launch(const AttnWideOp& op, cudaStream_t st)
{
    static std::atomic<uint64_t> attr_devs{0};
    const cudaError_t e = smem_limit_once(attr_devs, k_attn_wide<D>, kWSmem<D>);
    if (e != cudaSuccess)
        return e;
    launch_k(k_attn_wide<D>, op.grid, kWThreads, kWSmem<D>, st, op.tm, op.args);
    count_launch();
    return cudaGetLastError();
}

}  // namespace

bool attn_wide_prepare(AttnWideOp& op, const void* qkv, long ld, const AttnWideArgs& args, const char** err)
{
    op.ready = false;
    const int D = args.d;
    if ((D != 256 && D != 512) || args.n <= 0 || !args.out || (args.ldo & 7) || (args.ldo < D) ||
        (args.q_col | args.k_col | args.v_col) % 64 || args.q_col < 0 || args.k_col < 0 || args.v_col < 0 ||
        args.q_col + D > ld || args.k_col + D > ld || args.v_col + D > ld || (ld & 7) ||
        (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(args.out) & 15)) {
        *err = "attention_wide: head dim 256 or 512, q/k/v columns multiples of 64 inside rows of ld (a multiple of "
               "8), 16-byte aligned buffers";
        return false;
    }
    auto fn = wide_encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    // Rows of ld bf16 (q | k | v side by side), boxes of 64 columns x 128 rows with the 128-byte swizzle; rows past
    // n read as zeros.
    cuuint64_t dims[2] = {cuuint64_t(ld), cuuint64_t(args.n)};
    cuuint64_t strides[1] = {cuuint64_t(ld) * 2};
    cuuint32_t box[2] = {64, 128};
    cuuint32_t es[2] = {1, 1};
    if (fn(&op.tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(qkv), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        *err = "attention_wide: tensor map encoding failed";
        return false;
    }
    op.args = args;
    op.grid = dim3((args.n + kWTile - 1) / kWTile, 2, 1);
    op.ready = true;
    return true;
}

cudaError_t attn_wide_launch(const AttnWideOp& op, cudaStream_t st)
{
    if (!op.ready)
        return cudaErrorInvalidValue;
    return op.args.d == 512 ? wide_launch<512>(op, st) : wide_launch<256>(op, st);
}

}  // namespace mkb
