// Flash attention forward, head dim 64 or 128, on tcgen05 (see attention.cuh).
//
// One CTA per SM-sized work item: two 128-row query tiles (A and B) of one (sample, head) share every K/V tile.
// Three warpgroups:
//   warp 0     TMA: both Q tiles once, then K and V tiles of 128 keys into 2-stage rings (128-byte swizzle,
//              two 64-wide panels each)
//   warp 1     MMA, per KV tile j: O_A += P_A V, S_A = Q_A K_{j+1}^T, O_B += P_B V, S_B = Q_B K_{j+1}^T, with P read
//              from tensor memory. While one tile's softmax runs, the tensor pipe works on the other tile.
//   warps 2-3  idle (they complete the first warpgroup, which gives its registers to the softmax groups)
//   warps 4-7  softmax of tile A, warps 8-11 of tile B: one thread per query row holds its 128 scores in registers,
//              keeps a running max with lazy rescaling (O is rescaled only when a row's max grows by more than 2^8),
//              writes P = 2^(S - m) as bf16 over the first 64 columns of its S, and at the end stores O / l into the
//              output projection's input rows. At head dim 64 part of each row's exponentials run as a polynomial on
//              the FMA pipe to offload the SFU.
// TMEM columns: S_A [0, 128), S_B [128, 256), O_A [256, 384), O_B [384, 512).
#include "attention.cuh"
#include "gemm.cuh"
#include "sm100.cuh"
#include "common.cuh"
#include "launch.cuh"

#include <cudaTypedefs.h>
#include <cmath>
#include <cstdlib>
#include <mutex>

namespace mkb {

namespace {

constexpr int kThreads = 384;
// Registers per thread: the launch bound gives every thread 168 (3 warps share each SM sub-partition's 512 per
// lane); the control warpgroup drops to kRegsCtl and the two softmax warpgroups rise to kRegsSoftmax, enough to hold
// a row's 128 scores without spilling.
constexpr int kLaunchRegs = (65536 / kThreads) / 8 * 8;
constexpr int kRegsCtl = 56, kRegsSoftmax = 216;
static_assert(128 * kRegsCtl + 256 * kRegsSoftmax <= kThreads * kLaunchRegs, "register split exceeds the CTA pool");
static_assert(kRegsCtl + 2 * kRegsSoftmax <= 512, "register split exceeds a sub-partition");
constexpr int kTile = 128;                 // query rows per tile, keys per KV tile
constexpr int kPanel = kTile * 64 * 2;     // one 64-wide bf16 panel of 128 rows: 16 KB
template <int HD>
constexpr int kTileBytes = (HD / 64) * kPanel;  // a 128-row tile of one head: 16 KB (hd 64) or 32 KB (hd 128)
template <int HD>
constexpr int kSmem = 1024 + 6 * kTileBytes<HD> + 256;
constexpr uint32_t kTmemCols = 512;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// Score pair i of every 16-pair chunk with i % kEmuEvery == kEmuEvery - 1 takes 2^x from the FMA pipe (the packed
// two-lane polynomial) instead of the SFU; 0: none. At head dim 128 the SFU keeps up with the tensor pipe (moving
// 1/8, 1/4 or 1/3 of the exponentials measured 2-6% slower). At 64 the MMAs are half as long and 1/8 moves, spread
// through the row (162 us against 166 us at the 64^2 UNet shape for the same share as one block at the row's end,
// 167 us for 1/4).
template <int HD>
constexpr int kEmuEvery = HD == 128 ? 0 : 8;
// P published in two 64-key halves so P V of the first half starts while the second half's exponentials run: a
// gain at head dim 64 (where P V of a tile is half as long), a loss at 128 (measured 440 -> 464 and 1057 -> 1012
// TFLOP/s), so only there. Unsplit, the whole P is published on the second half's barrier.
template <int HD>
constexpr bool kSplitP = HD == 64;

__device__ __forceinline__ float ex2(float x)
{
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32])
{
    uint32_t a[16], b[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        a[i] = r[i];
        b[i] = r[16 + i];
    }
    tmem_st16(taddr, a);
    tmem_st16(taddr + 16, b);
}

// PAIR (head dim 128, MKB_ATTN_PAIR=1): CTAs run as clusters of two over the same (sample, head), each with its own two
// query tiles, and the leader issues every MMA for both as 256-row cta_group::2 MMAs: each CTA loads half of every key
// tile (64 keys, by rows) and half of every V tile (64 of the 128 columns), so per SM the K and V tiles cross shared
// memory at half the bytes. The follower's softmax signals P on the leader's barrier; the leader's commits reach both
// CTAs. Measured at the config-2 shape it is slower than one CTA per tile pair (832 against 1093 TFLOP/s; 920 with a
// quarter of the exponentials on the FMA pipe): the two CTAs' softmax phases now gate every MMA of both, and the
// exponentials, not shared memory, set the pace. It stays as an option, tested for parity.
template <int HD, bool PAIR>
__global__ void __launch_bounds__(kThreads, 1)
    k_attn(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
           const __grid_constant__ CUtensorMap tv, const AttnArgs a)
{
    static_assert(!PAIR || HD == 128, "CTA pairs split V by 64-column panels: head dim 128 only");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int TB = kTileBytes<HD>;
    uint8_t* sQ = smem;           // [2 tiles][TB]
    uint8_t* sK = smem + 2 * TB;  // [2 stages][TB]
    uint8_t* sV = smem + 4 * TB;  // [2 stages][TB]
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * TB);
    uint64_t* q_full = bars + 0;
    uint64_t* k_full = bars + 1;    // [2]
    uint64_t* k_empty = bars + 3;   // [2]
    uint64_t* v_full = bars + 5;    // [2]
    uint64_t* v_empty = bars + 7;   // [2]
    uint64_t* s_full = bars + 9;    // [2 tiles]
    uint64_t* p_full = bars + 11;   // [2 tiles][2 halves of the keys]
    uint64_t* o_done = bars + 15;   // [2 tiles]
    uint64_t* drain = bars + 17;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = blockIdx.x * 2 * kTile, h = blockIdx.y, b = blockIdx.z;
    const int bh = b * a.H + h;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0;
    const bool leader = rank == 0;

    // Keys this CTA (pair) needs: when its query rows are all condition rows (causal among themselves), keys up to
    // the last row's position.
    int n_keys = a.Lk;
    if (a.mask == kMaskCondCausal) {
        const int q_end = PAIR ? ((blockIdx.x | 1) + 1) * 2 * kTile : q0 + 2 * kTile;
        const int last_pos = a.q_pos0 + min(q_end, a.Lq) - 1;
        if (last_pos < a.cond_len)
            n_keys = min(a.Lk, last_pos + 1);
    }
    const int nkv = (n_keys + kTile - 1) / kTile;
    // Key tile taken at step j: j0 + j, wrapping round (j0 = 0 unless other ranks' shards arrive during the launch).
    const int j0 = a.own_shard >= 0 && a.rotate ? a.own_shard * (a.kv_shard_rows / kTile) : 0;
    const auto key_tile = [&](int j) { return j + j0 < nkv ? j + j0 : j + j0 - nkv; };

    if (threadIdx.x == 0) {
        mbar_init(q_full, 1);
        for (int i = 0; i < 2; ++i) {
            mbar_init(&k_full[i], 1);
            mbar_init(&k_empty[i], 1);
            mbar_init(&v_full[i], 1);
            mbar_init(&v_empty[i], 1);
            mbar_init(&s_full[i], 1);
            mbar_init(&p_full[2 * i], PAIR ? 256 : 128);  // (pairs: the leader's, both CTAs' softmax threads)
            mbar_init(&p_full[2 * i + 1], PAIR ? 256 : 128);
            mbar_init(&o_done[i], 1);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tq);
        prefetch_tmap(&tk);
        prefetch_tmap(&tv);
    }
    grid_dep_wait();  // before TMEM allocation and the first global access
    if (warp == 1) {
        if constexpr (PAIR) {
            tmem_alloc_pair(tmem_slot, kTmemCols);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, kTmemCols);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR)
        cluster_sync_all();  // both CTAs' barriers exist before either signals the other's
    tc_fence_after();
    grid_dep_launch();
    const uint32_t tmem = *tmem_slot;

    if (warp < 4)
        regs_decrease<kRegsCtl>();
    if (warp == 0) {
        if (lane == 0) {
            int issued_k = 0, issued_v = 0;
            bool ok = true, q_issued = PAIR;
            int arrived = a.own_shard;  // the shard whose arrival was last confirmed
            const unsigned long long want = a.own_shard >= 0 ? *a.shard_expect : 0;
            // Row and plane of query tile t (shards never split a tile: q_shard_rows is a multiple of 128).
            const auto q_at = [&](int t, int* plane) {
                int row = a.q_row0 + q0 + t * kTile;
                *plane = bh;
                if (a.q_shard_rows > 0) {
                    const int g = row / a.q_shard_rows;
                    row -= g * a.q_shard_rows;
                    *plane = g * a.q_plane_stride + bh;
                }
                return row;
            };
            if constexpr (PAIR) {
                if (leader)
                    mbar_arrive_expect_tx(q_full, 4 * TB);  // both CTAs' two tiles
                for (int t = 0; t < 2; ++t) {
                    int plane;
                    const int row = q_at(t, &plane);
                    for (int pn = 0; pn < HD / 64; ++pn)
                        tma_load_3d_pair(sQ + t * TB + pn * kPanel, &tq, q_full, pn * 64, row, plane);
                }
            } else {
                // Query rows stored by other ranks during the launch: each tile's shard once its flag is up.
                if (a.own_shard >= 0 && a.q_shard_rows > 0)
                    for (int t = 0; t < 2 && ok; ++t) {
                        const int gq = (a.q_row0 + q0 + t * kTile) / a.q_shard_rows;
                        if (gq != a.own_shard && q0 + t * kTile < a.Lq)
                            ok = wait_flag_ge(a.shard_ready + gq, want, a.status, kErrShardWait, abort_flag);
                    }
                if (ok) {
                    mbar_arrive_expect_tx(q_full, 2 * TB);
                    for (int t = 0; t < 2; ++t) {
                        int plane;
                        const int row = q_at(t, &plane);
                        for (int pn = 0; pn < HD / 64; ++pn)
                            tma_load_3d(sQ + t * TB + pn * kPanel, &tq, q_full, pn * 64, row, plane);
                    }
                    q_issued = true;
                }
            }
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j & 1;
                const uint32_t ph = (j >> 1) & 1;
                if (!mbar_wait(&k_empty[st], ph ^ 1, a.status, kErrAttnWait, abort_flag)) {
                    ok = false;
                    break;
                }
                // Row and plane of the key tile (shards never split a tile: kv_shard_rows is a multiple of 128).
                int krow = key_tile(j) * kTile, kplane = bh;
                if (a.kv_shard_rows > 0) {
                    const int g = krow / a.kv_shard_rows;
                    krow -= g * a.kv_shard_rows;
                    kplane = g * a.kv_plane_stride + bh;
                    if (a.own_shard >= 0 && g != arrived && g != a.own_shard) {  // another rank's: once landed
                        if (!wait_flag_ge(a.shard_ready + g, want, a.status, kErrShardWait, abort_flag)) {
                            ok = false;
                            break;
                        }
                        arrived = g;
                    }
                }
                if constexpr (PAIR) {  // this CTA's 64 keys of the tile; the leader's barrier counts both halves
                    if (leader)
                        mbar_arrive_expect_tx(&k_full[st], TB);
                    for (int pn = 0; pn < HD / 64; ++pn)
                        tma_load_3d_pair(sK + st * TB + pn * (kPanel / 2), &tk, &k_full[st], pn * 64,
                                         krow + 64 * int(rank), kplane);
                } else {
                    mbar_arrive_expect_tx(&k_full[st], TB);
                    for (int pn = 0; pn < HD / 64; ++pn)
                        tma_load_3d(sK + st * TB + pn * kPanel, &tk, &k_full[st], pn * 64, krow, kplane);
                }
                ++issued_k;
                if (!mbar_wait(&v_empty[st], ph ^ 1, a.status, kErrAttnWait, abort_flag)) {
                    ok = false;
                    break;
                }
                if constexpr (PAIR) {  // this CTA's 64 columns of V
                    if (leader)
                        mbar_arrive_expect_tx(&v_full[st], TB);
                    tma_load_3d_pair(sV + st * TB, &tv, &v_full[st], 64 * int(rank), krow, kplane);
                } else {
                    mbar_arrive_expect_tx(&v_full[st], TB);
                    for (int pn = 0; pn < HD / 64; ++pn)
                        tma_load_3d(sV + st * TB + pn * kPanel, &tv, &v_full[st], pn * 64, krow, kplane);
                }
                ++issued_v;
            }
            // Let the loads already issued land before the CTA can exit (a pair's loads complete on the leader's
            // barriers, which only the leader can wait on: the cluster barrier at the end keeps both CTAs alive).
            if (!ok && !PAIR) {
                if (q_issued)
                    mbar_wait(q_full, 0, a.status, kErrWaitDrain, nullptr);
                for (int j = issued_k > 2 ? issued_k - 2 : 0; j < issued_k; ++j)
                    mbar_wait(&k_full[j & 1], (j >> 1) & 1, a.status, kErrWaitDrain, nullptr);
                for (int j = issued_v > 2 ? issued_v - 2 : 0; j < issued_v; ++j)
                    mbar_wait(&v_full[j & 1], (j >> 1) & 1, a.status, kErrWaitDrain, nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && leader) {
            constexpr int kM = PAIR ? 256 : 128;  // a pair's MMAs cover both CTAs' 128 rows
            constexpr uint32_t idesc_s = idesc_bf16_f32(kM, 128, 0, 0);
            constexpr uint32_t idesc_o = idesc_bf16_f32(kM, HD, 0, 1);  // V is MN-major (head dim contiguous)
            const auto commit = [](uint64_t* bar) {
                if constexpr (PAIR)
                    mma_commit_pair(bar);
                else
                    mma_commit(bar);
            };
            const uint32_t q_addr = smem_u32(sQ), k_addr = smem_u32(sK), v_addr = smem_u32(sV);
            // Issue order per key tile j: PV_A(j), S_A(j+1), PV_B(j), S_B(j+1). Each tile's next S follows its own
            // P V directly, so tile A's softmax overlaps tile B's two MMAs and the other way round. S_t(j+1)
            // overwrites the TMEM columns P_t(j) occupies; both come from this thread, and the tensor pipe executes
            // one CTA's MMAs in issue order, so P_t(j) is read before it is overwritten. The commit after S_t(j+1)
            // also covers PV_t(j), so when a softmax warp sees s_full its O accumulator is settled for rescaling.
            const auto issue_s = [&](int t, int st) {
#pragma unroll
                for (int k = 0; k < HD / 16; ++k) {
                    const uint32_t off = (k >> 2) * kPanel + (k & 3) * 32;
                    if constexpr (PAIR)  // each CTA's K half: 64-row panels
                        mma_bf16_ss_pair(tmem + t * 128, desc_kmajor_sw128(q_addr + t * TB + off),
                                         desc_kmajor_sw128(k_addr + st * TB + (k >> 2) * (kPanel / 2) + (k & 3) * 32),
                                         idesc_s, k > 0);
                    else
                        mma_bf16_ss(tmem + t * 128, desc_kmajor_sw128(q_addr + t * TB + off),
                                    desc_kmajor_sw128(k_addr + st * TB + off), idesc_s, k > 0);
                }
                commit(&s_full[t]);
            };
            bool ok = mbar_wait(q_full, 0, a.status, kErrAttnWait, abort_flag);
            if (ok && nkv > 0) {
                ok = mbar_wait(&k_full[0], 0, a.status, kErrAttnWait, abort_flag);
                if (ok) {
                    tc_fence_after();
                    issue_s(0, 0);
                    issue_s(1, 0);
                    commit(&k_empty[0]);
                }
            }
            for (int j = 0; j < nkv && ok; ++j) {
                const int st = j & 1, st1 = (j + 1) & 1;
                const bool next = j + 1 < nkv;
                if (!mbar_wait(&v_full[st], (j >> 1) & 1, a.status, kErrAttnWait, abort_flag))
                    break;
                if (next && !mbar_wait(&k_full[st1], ((j + 1) >> 1) & 1, a.status, kErrAttnWait, abort_flag))
                    break;
                for (int t = 0; t < 2 && ok; ++t) {
                    for (int half = kSplitP<HD> ? 0 : 1; half < 2 && ok; ++half) {
                        if (!mbar_wait(&p_full[2 * t + half], j & 1, a.status, kErrAttnWait, abort_flag)) {
                            ok = false;
                            break;
                        }
                        tc_fence_after();
                        // 16 keys per step: P columns 8k.., V rows 16k.. (two 8-row atoms).
#pragma unroll
                        for (int k = kSplitP<HD> ? 4 * half : 0; k < 4 * half + 4; ++k) {
                            if constexpr (PAIR)  // each CTA's 64 columns of V: one panel
                                mma_bf16_ts_pair(tmem + 256 + t * HD, tmem + t * 128 + 8 * k,
                                                 desc_mnmajor_sw128(v_addr + st * TB + k * 2048, kPanel, 1024),
                                                 idesc_o, (j > 0) || (k > 0));
                            else
                                mma_bf16_ts(tmem + 256 + t * HD, tmem + t * 128 + 8 * k,
                                            desc_mnmajor_sw128(v_addr + st * TB + k * 2048, kPanel, 1024), idesc_o,
                                            (j > 0) || (k > 0));
                        }
                    }
                    if (!ok)
                        break;
                    commit(&o_done[t]);
                    if (next)
                        issue_s(t, st1);
                }
                if (!ok)
                    break;
                commit(&v_empty[st]);
                if (next)
                    commit(&k_empty[st1]);
            }
            commit(drain);  // arrives once every MMA issued above has completed
            mbar_wait(drain, 0, a.status, kErrWaitDrain, nullptr);
        }
    } else if (warp >= 4) {
        regs_increase<kRegsSoftmax>();
        const int t = (warp - 4) >> 2;  // query tile of this softmax warp group
        const int quarter = warp & 3;
        const int r = quarter * 32 + lane;
        const uint32_t t_lane = tmem + (uint32_t(quarter * 32) << 16);
        const uint32_t col_s = t * 128, col_o = 256 + t * HD;
        const int qrow = q0 + t * kTile + r;
        const int qpos = a.q_pos0 + qrow;
        const bool text_query = a.mask == kMaskCondCausal && qpos < a.cond_len;
        const int key_limit = text_query ? min(a.Lk, qpos + 1) : a.Lk;  // a condition row: keys up to its own
        const float sc = a.scale_log2;
        float m_used = -INFINITY, l = 0.0f;
        bool ok = true;
        for (int j = 0; j < nkv; ++j) {
            if (!mbar_wait(&s_full[t], j & 1, a.status, kErrAttnWait, abort_flag)) {
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
            const int valid = min(kTile, key_limit - key_tile(j) * kTile);  // keys [0, valid) of the tile are visible
            if (valid < kTile) {
#pragma unroll
                for (int i = 0; i < 128; ++i)
                    if (i >= valid)
                        s[i] = __float_as_uint(-INFINITY);
            }
            // Row max as 8 independent chains of 3-input max (a single chain would serialize 64 dependent ops).
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
            const bool need = mx > m_used + kRescaleThreshold;
            if (__any_sync(0xffffffffu, need)) {
                const float m_new = need ? mx : m_used;
                const float f = ex2(m_used - m_new);  // 0 on the first tile
                l *= f;
                if (j > 0) {
#pragma unroll 1
                    for (int c = 0; c < HD / 32; ++c) {
                        uint32_t o[32];
                        tmem_ld32(t_lane + col_o + c * 32, o);
                        tmem_wait_ld();
#pragma unroll
                        for (int i = 0; i < 32; ++i)
                            o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
                        tmem_st32(t_lane + col_o + c * 32, o);
                    }
                }
                m_used = m_new;
            }
            // x = s * scale - m for two scores per packed FMA; the row sum in 4 packed accumulators.
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
                    constexpr int kEvery = kEmuEvery<HD> ? kEmuEvery<HD> : 1 << 30;
                    if (i % kEvery == kEvery - 1) {
                        e = ex2_poly2(x);
                    } else {
                        e.x = ex2(x.x);
                        e.y = ex2(x.y);
                    }
                    ls[i & 3] = fadd2(ls[i & 3], e);
                    p[i] = pack_bf16x2(e.x, e.y);
                }
                tmem_st16(t_lane + col_s + c * 16, p);
                if (c == 3 || (kSplitP<HD> && c == 1)) {  // keys up to 64 (c + 1) / 2 published
                    tmem_wait_st();
                    tc_fence_before();
                    if (PAIR && !leader)  // the leader's barrier counts both CTAs' rows
                        mbar_arrive_cluster(map_to_cta(smem_u32(&p_full[2 * t + c / 2]), 0));
                    else
                        mbar_arrive(&p_full[2 * t + c / 2]);
                }
            }
            const float2 l01 = fadd2(fadd2(ls[0], ls[1]), fadd2(ls[2], ls[3]));
            l += l01.x + l01.y;
        }
        if (ok && nkv > 0 && mbar_wait(&o_done[t], (nkv - 1) & 1, a.status, kErrAttnWait, abort_flag)) {
            tc_fence_after();
            const float inv = l > 0.0f ? 1.0f / l : 0.0f;
            const bool row_ok = qrow < a.Lq;
            __nv_bfloat16* dst = nullptr;
            if (row_ok) {
                if (a.out_shard_rows > 0) {
                    const int g = qpos / a.out_shard_rows, i = qpos - g * a.out_shard_rows;
                    const AttnOutShard& e = a.out_shards[g];
                    dst = i < e.text_rows ? e.txt + (long(b) * e.text_rows + i) * a.ld0
                                          : e.img + (long(b) * (a.out_shard_rows - e.text_rows) + i - e.text_rows) * a.ld0;
                } else {
                    dst = qpos < a.split ? a.out0 + (long(b) * a.rows0 + qpos) * a.ld0
                                         : a.out1 + (long(b) * a.rows1 + (qpos - a.split)) * a.ld1;
                }
                dst += h * HD;
            }
#pragma unroll 1
            for (int c = 0; c < HD / 32; ++c) {
                uint32_t o[32];
                tmem_ld32(t_lane + col_o + c * 32, o);
                tmem_wait_ld();
                if (row_ok) {
                    uint4* d = reinterpret_cast<uint4*>(dst + c * 32);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        d[i] = make_uint4(pack_bf16x2(__uint_as_float(o[8 * i]) * inv, __uint_as_float(o[8 * i + 1]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * i + 2]) * inv, __uint_as_float(o[8 * i + 3]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * i + 4]) * inv, __uint_as_float(o[8 * i + 5]) * inv),
                                          pack_bf16x2(__uint_as_float(o[8 * i + 6]) * inv, __uint_as_float(o[8 * i + 7]) * inv));
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if constexpr (PAIR)
        cluster_sync_all();  // the leader's MMAs read this CTA's shared memory and tensor memory until here
    if (warp == 1) {
        tc_fence_after();
        if constexpr (PAIR)
            tmem_dealloc_pair(tmem, kTmemCols);
        else
            tmem_dealloc(tmem, kTmemCols);
    }
}

bool attn_pairs_enabled()
{
    static const bool on = [] {
        const char* v = std::getenv("MKB_ATTN_PAIR");
        return v && v[0] == '1';
    }();
    return on;
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

// Head-major [BH][rows][128] bf16 as a 3-D map, box 64 x box_rows x 1 with the 128-byte swizzle; rows past `rows` of
// a head read as zeros.
bool make_heads_map(CUtensorMap* m, const void* p, int rows, int bh, int hd, const char** err, int box_rows = 128)
{
    auto fn = encode_fn();
    if (!fn) {
        *err = "cuTensorMapEncodeTiled unavailable";
        return false;
    }
    if (reinterpret_cast<uintptr_t>(p) & 15) {
        *err = "attention: q/k/v must be 16-byte aligned";
        return false;
    }
    cuuint64_t dims[3] = {cuuint64_t(hd), cuuint64_t(rows), cuuint64_t(bh)};
    cuuint64_t strides[2] = {cuuint64_t(hd) * 2, cuuint64_t(rows) * hd * 2};
    cuuint32_t box[3] = {64, cuuint32_t(box_rows), 1};
    cuuint32_t es[3] = {1, 1, 1};
    if (fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(p), dims, strides, box, es,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS) {
        *err = "attention: tensor map encoding failed";
        return false;
    }
    return true;
}

}  // namespace

bool attn_prepare(AttnOp& op, const void* q, int Lq_rows, const void* k, const void* v, int Lk_rows,
                  const AttnArgs& args, const char** err)
{
    op.ready = false;
    if (args.B <= 0 || args.H <= 0 || args.Lq <= 0 || args.Lk <= 0 || args.q_row0 < 0 ||
        (args.q_shard_rows <= 0 && Lq_rows < args.q_row0 + args.Lq) || Lk_rows < args.Lk) {
        *err = "attention: bad sizes";
        return false;
    }
    if (args.out_shard_rows > 0) {
        if (!args.out_shards || (args.ld0 & 7) || args.q_pos0 < 0 || args.ld0 < long(args.H) * args.head_dim) {
            *err = "attention: output shards need their table and ld0 a multiple of 8 covering the heads";
            return false;
        }
    } else {
        const bool text_rows = args.q_pos0 < args.split;  // some query rows route to out0
        if (!args.out1 || (text_rows && !args.out0) || (args.ld0 & 7) || (args.ld1 & 7)) {
            *err = "attention: outputs missing or leading dimensions not multiples of 8";
            return false;
        }
        if ((text_rows && args.rows0 < args.split) || args.q_pos0 < 0 ||
            args.q_pos0 + args.Lq - args.split > args.rows1) {
            *err = "attention: output rows do not cover the query positions";
            return false;
        }
    }
    if (args.mask == kMaskCondCausal && args.cond_len <= 0) {
        *err = "attention: condition-causal mask needs cond_len > 0";
        return false;
    }
    const int bh = args.B * args.H;
    if (args.head_dim != 64 && args.head_dim != 128) {
        *err = "attention: head dim must be 64 or 128";
        return false;
    }
    const int hd = args.head_dim;
    int kv_rows = Lk_rows, kv_planes = bh;
    if (args.kv_shard_rows > 0) {
        if (args.kv_shard_rows % 128 || args.kv_plane_stride < bh) {
            *err = "attention: K/V shards need a multiple of 128 rows and a plane stride >= B * H";
            return false;
        }
        const int shards = (args.Lk + args.kv_shard_rows - 1) / args.kv_shard_rows;
        kv_rows = args.kv_shard_rows;
        kv_planes = (shards - 1) * args.kv_plane_stride + bh;
    }
    if (args.own_shard >= 0 &&
        (args.kv_shard_rows <= 0 || args.mask != kMaskNone || !args.shard_ready || !args.shard_expect ||
         long(args.own_shard) * args.kv_shard_rows >= args.Lk || (reinterpret_cast<uintptr_t>(args.shard_ready) & 7))) {
        *err = "attention: arriving shards need K/V shards, no mask, 8-byte aligned flags and own_shard inside Lk";
        return false;
    }
    int q_rows = Lq_rows, q_planes = bh;
    if (args.q_shard_rows > 0) {
        if (args.q_shard_rows % 128 || args.q_plane_stride < bh || args.q_row0 != 0 || Lq_rows < args.q_shard_rows) {
            *err = "attention: query shards need a multiple of 128 rows, q_row0 0 and a plane stride >= B * H";
            return false;
        }
        const int shards = (args.Lq + args.q_shard_rows - 1) / args.q_shard_rows;
        q_rows = args.q_shard_rows;
        q_planes = (shards - 1) * args.q_plane_stride + bh;
    }
    // CTA pairs for head dim 128 (MKB_ATTN_PAIR=0: one CTA per pair of query tiles throughout); not with query
    // tiles that arrive during the launch.
    op.pair = hd == 128 && attn_pairs_enabled() && !(args.own_shard >= 0 && args.q_shard_rows > 0);
    if (!make_heads_map(&op.tq, q, q_rows, q_planes, hd, err) ||
        !make_heads_map(&op.tk, k, kv_rows, kv_planes, hd, err, op.pair ? 64 : 128) ||
        !make_heads_map(&op.tv, v, kv_rows, kv_planes, hd, err))
        return false;
    op.args = args;
    const int blocks = (args.Lq + 2 * kTile - 1) / (2 * kTile);
    op.grid = dim3(op.pair ? (blocks + 1) / 2 * 2 : blocks, args.H, args.B);
    op.ready = true;
    return true;
}

namespace {

// Set-up of a kernel instance: a one-time check that the compiled launch register count holds the warpgroups'
// register split (otherwise the softmax groups' increase could never be granted), and its shared memory size on
// each device it runs on.
template <int HD, bool PAIR>
cudaError_t attn_setup()
{
    static const cudaError_t regs = [] {
        cudaFuncAttributes fa{};
        cudaError_t e = cudaFuncGetAttributes(&fa, k_attn<HD, PAIR>);
        if (e != cudaSuccess)
            return e;
        return fa.numRegs * kThreads < 128 * kRegsCtl + 256 * kRegsSoftmax ? cudaErrorInvalidConfiguration
                                                                          : cudaSuccess;
    }();
    if (regs != cudaSuccess)
        return regs;
    static std::atomic<uint64_t> attr_devs{0};
    return smem_limit_once(attr_devs, k_attn<HD, PAIR>, kSmem<HD>);
}

}  // namespace

cudaError_t attn_launch(const AttnOp& op, cudaStream_t st)
{
    if (!op.ready)
        return cudaErrorInvalidValue;
    if (op.args.head_dim == 64) {
        cudaError_t e = attn_setup<64, false>();
        if (e != cudaSuccess)
            return e;
        launch_k(k_attn<64, false>, op.grid, kThreads, kSmem<64>, st, op.tq, op.tk, op.tv, op.args);
    } else {
        cudaError_t e = op.pair ? attn_setup<128, true>() : attn_setup<128, false>();
        if (e != cudaSuccess)
            return e;
        if (op.pair)
            launch_k_pairs(k_attn<128, true>, op.grid, kThreads, kSmem<128>, st, op.tq, op.tk, op.tv, op.args);
        else
            launch_k(k_attn<128, false>, op.grid, kThreads, kSmem<128>, st, op.tq, op.tk, op.tv, op.args);
    }
    count_launch();
    return cudaGetLastError();
}

}  // namespace mkb
