// Thin wrappers over the sm_100a instructions the kernels use: mbarriers with bounded waits, TMA tile loads,
// tcgen05 tensor-memory allocation, MMA issue, commit and loads, and the shared-memory matrix descriptors.
//
// Every wait here is bounded: a wait that has not completed after kWaitNs of wall time sets a bit in the launch's
// status word and returns false, so a broken pipeline ends the kernel with an error the host reads instead of a hang.
#pragma once

#include <cstdint>
#include <cuda_bf16.h>

namespace mkb {

// Status bits written by kernels (the host reads them back after a step; 0 = success).
enum : uint32_t {
    kErrWaitFull = 1u << 0,      // consumer of a shared-memory stage gave up waiting for its TMA load
    kErrWaitEmpty = 1u << 1,     // producer gave up waiting for a stage to be released
    kErrWaitAccFull = 1u << 2,   // epilogue gave up waiting for an accumulator
    kErrWaitAccEmpty = 1u << 3,  // MMA issuer gave up waiting for the epilogue to drain an accumulator
    kErrWaitDrain = 1u << 4,     // final drain of in-flight copies / MMAs timed out
    kErrAttnWait = 1u << 5,      // attention pipeline wait timed out
    kErrShape = 1u << 6,         // a kernel was launched with a shape it does not support
    kErrWaitEpiLoad = 1u << 7,   // GEMM epilogue gave up waiting for its residual box
    kErrShardWait = 1u << 8,     // attention gave up waiting for another rank's K/V shard to arrive
};

constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s: far above any legitimate stage wait

__device__ __forceinline__ uint64_t globaltimer_ns()
{
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p)
{
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Packed two-lane fp32 arithmetic: one instruction for both lanes.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c)
{
    uint64_t ra = *reinterpret_cast<uint64_t*>(&a), rb = *reinterpret_cast<uint64_t*>(&b),
             rc = *reinterpret_cast<uint64_t*>(&c), rd;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(rd) : "l"(ra), "l"(rb), "l"(rc));
    return *reinterpret_cast<float2*>(&rd);
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b)
{
    uint64_t ra = *reinterpret_cast<uint64_t*>(&a), rb = *reinterpret_cast<uint64_t*>(&b), rd;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(rd) : "l"(ra), "l"(rb));
    return *reinterpret_cast<float2*>(&rd);
}

// 2^x for two lanes on the FMA pipe with packed f32x2 arithmetic: x = n + f with n = round(x), f in [-1/2, 1/2]; 2^f
// by the degree-3 polynomial of least maximum relative error on that interval (a minimax fit by the Remez exchange
// algorithm, tests/ex2_fit.py; 7.5e-5, below bf16's 3.9e-3; tests/test_ex2_poly_cpu.py checks the bound), 2^n added
// to the exponent bits. Arguments below -126 flush to 0 like ex2.approx.ftz.
__device__ __forceinline__ float2 ex2_poly2(float2 x)
{
    x.x = fmaxf(x.x, -126.0f);
    x.y = fmaxf(x.y, -126.0f);
    const float2 t = fadd2(x, make_float2(12582912.0f, 12582912.0f));
    const float2 n = fadd2(t, make_float2(-12582912.0f, -12582912.0f));
    const float2 f = ffma2(n, make_float2(-1.0f, -1.0f), x);
    float2 p = ffma2(make_float2(0.055171459913253784f, 0.055171459913253784f), f,
                     make_float2(0.2426108568906784f, 0.2426108568906784f));
    p = ffma2(p, f, make_float2(0.6932609677314758f, 0.6932609677314758f));
    p = ffma2(p, f, make_float2(0.9999281167984009f, 0.9999281167984009f));
    return make_float2(__int_as_float(__float_as_int(p.x) + ((__float_as_int(t.x) - 0x4B400000) << 23)),
                       __int_as_float(__float_as_int(p.y) + ((__float_as_int(t.y) - 0x4B400000) << 23)));
}

__device__ __forceinline__ float fmax3(float a, float b, float c)
{
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Waits until the 64-bit flag in global memory (written by another GPU's copy engine) reaches `want`: an acquire
// load at system scope, then a proxy fence so that TMA loads issued after the return see the data written before
// the flag. Gives up after kWaitNs (sets `err_bit` and *abort), at once when *abort is set by another role of the
// CTA, and when `err_bit` is already set in *status (another CTA gave up on the same flag).
__device__ __forceinline__ bool wait_flag_ge(const unsigned long long* flag, unsigned long long want,
                                             uint32_t* status, uint32_t err_bit, volatile int* abort)
{
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 0;; ++it) {
        unsigned long long v;
        asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
        if (v >= want) {
            asm volatile("fence.proxy.async.global;" ::: "memory");
            return true;
        }
        const bool others = status && (*reinterpret_cast<volatile uint32_t*>(status) & err_bit);
        if ((abort && *abort) || others || globaltimer_ns() - t0 > kWaitNs) {
            if (status && !others)
                atomicOr(status, err_bit);
            if (abort)
                *abort = 1;
            return false;
        }
        __nanosleep(128);
    }
}

// ---------------------------------------------------------------- mbarrier

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count)
{
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init()
{
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar)
{
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes)
{
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar_addr, uint32_t parity)
{
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar_addr), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for the phase with the given parity to complete. Returns false (and sets `err_bit` in *status) after
// kWaitNs, or at once if *abort is already set by another role of the same CTA.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* status, uint32_t err_bit,
                                          volatile int* abort)
{
    const uint32_t a = smem_u32(bar);
    if (mbar_try_wait(a, parity))
        return true;
    const uint64_t t0 = globaltimer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(a, parity))
            return true;
        if ((it & 255) == 0) {
            if (abort && *abort)
                return false;
            if (globaltimer_ns() - t0 > kWaitNs) {
                if (status)
                    atomicOr(status, err_bit);
                if (abort)
                    *abort = 1;
                return false;
            }
        }
    }
}

// ---------------------------------------------------------------- TMA

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1)
{
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2)
{
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2, int c3)
{
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
        "[%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap)
{
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// Shared -> global tensor copies, tracked as bulk groups of the issuing thread. The store writes the box; the
// reduce adds it element-wise into global memory (the tensor map's element type). Boxes that reach past the
// tensor's extent are clipped.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int c0, int c1)
{
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}

__device__ __forceinline__ void tma_store_4d(const void* tmap, const void* src, int c0, int c1, int c2, int c3)
{
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
                 : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d(const void* tmap, const void* src, int c0, int c1)
{
    asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}

__device__ __forceinline__ void tma_reduce_add_4d(const void* tmap, const void* src, int c0, int c1, int c2, int c3)
{
    asm volatile(
        "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(tmap),
        "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }

// Waits until at most N of this thread's bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read()
{
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}

// Waits until all of this thread's bulk groups have completed (their global writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// Orders this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads of them.
__device__ __forceinline__ void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05

// One full warp allocates `ncols` TMEM columns (power of two, >= 32); the base address lands in *dst (shared).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Per-warpgroup register reallocation. Every warp of a warpgroup executes the same one. An increase waits until the
// registers are free in the CTA's pool, which holds (threads x registers at launch): the kernels that use these
// assert at compile time that their split fits, and the host checks the compiled launch count before launching.
template <uint32_t N>
__device__ __forceinline__ void regs_decrease()
{
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}
template <uint32_t N>
__device__ __forceinline__ void regs_increase()
{
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 inputs, fp32 accumulate). Single thread.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: the A operand (M rows x K) read from tensor memory. Single thread.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on *bar when every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* bar)
{
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane (base lane + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

// 32 lanes x 16 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}

// 32 lanes x 16 columns store (the thread's lane, columns [col, col+16)).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16])
{
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte swizzle (rows of 64 bf16,
// 8-row atoms of 1024 bytes one after another). `addr` is the shared address of the first element the MMA reads;
// the tile base must be 1024-byte aligned, and K steps inside an atom add 32 bytes per 16 elements.
__device__ __forceinline__ uint64_t desc_kmajor_sw128(uint32_t addr)
{
    uint64_t d = 0;
    d |= uint64_t((addr >> 4) & 0x3FFF);         // start address
    d |= uint64_t(1) << 16;                      // leading byte offset (unused for swizzled K-major)
    d |= uint64_t(1024 >> 4) << 32;              // stride byte offset: 8-row atom pitch
    d |= uint64_t(1) << 46;                      // descriptor version (sm_100)
    d |= uint64_t(2) << 61;                      // layout: 128-byte swizzle
    return d;
}

// Descriptor for an MN-major operand (N contiguous) stored with the 128-byte swizzle: the tile is a sequence of
// 64-element-wide column panels; each panel holds rows of 64 N-values (128 bytes) for consecutive K, 8-row atoms
// of 1024 bytes. `lbo` is the byte distance between panels along N, `sbo` the distance between 8-row K groups.
__device__ __forceinline__ uint64_t desc_mnmajor_sw128(uint32_t addr, uint32_t lbo, uint32_t sbo)
{
    uint64_t d = 0;
    d |= uint64_t((addr >> 4) & 0x3FFF);
    d |= uint64_t((lbo >> 4) & 0x3FFF) << 16;
    d |= uint64_t((sbo >> 4) & 0x3FFF) << 32;
    d |= uint64_t(1) << 46;
    d |= uint64_t(2) << 61;
    return d;
}

// Instruction descriptor of kind::f16 with bf16 A and B, fp32 accumulator. a_mn / b_mn: operand is MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn = 0, int b_mn = 0)
{
    return (1u << 4)                   // D format: f32
           | (1u << 7)                 // A format: bf16
           | (1u << 10)                // B format: bf16
           | (uint32_t(a_mn) << 15)    // A major
           | (uint32_t(b_mn) << 16)    // B major
           | (uint32_t(N >> 3) << 17)  // N / 8
           | (uint32_t(M >> 4) << 24); // M / 16
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)

__device__ __forceinline__ uint32_t cluster_ctarank()
{
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of the same offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t smem_addr, uint32_t rank)
{
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
    return r;
}

// Arrive on an mbarrier given by its shared::cluster address (possibly in the peer CTA).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr)
{
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

__device__ __forceinline__ void cluster_sync_all()
{
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// TMA load of this CTA's part of a pair tile, its completion counted on the pair leader's mbarrier (the barrier's
// shared address with the peer bit cleared).
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const void* tmap, uint64_t* bar, int c0, int c1)
{
    const uint32_t leader_bar = map_to_cta(smem_u32(bar), 0);
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(leader_bar), "r"(c0), "r"(c1)
        : "memory");
}

__device__ __forceinline__ void tma_load_4d_pair(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                                                 int c3)
{
    const uint32_t leader_bar = map_to_cta(smem_u32(bar), 0);
    asm volatile(
        "cp.async.bulk.tensor.4d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(leader_bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
        : "memory");
}

__device__ __forceinline__ void tma_load_3d_pair(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2)
{
    const uint32_t leader_bar = map_to_cta(smem_u32(bar), 0);
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
        "%4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(leader_bar), "r"(c0), "r"(c1), "r"(c2)
        : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst, uint32_t ncols)
{
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair()
{
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols)
{
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem of both CTAs] (+)= A (128 rows in each CTA) * B (N/2 rows in each CTA)^T: one 256 x N x 16 MMA issued by the
// pair leader.
__device__ __forceinline__ void mma_bf16_ss_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The same with A from tensor memory (each CTA's 128 rows in its own TMEM at a_tmem).
__device__ __forceinline__ void mma_bf16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                 uint32_t accumulate)
{
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive once on the mbarrier at this offset in both CTAs of the pair when the leader's MMAs so far complete.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar)
{
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(uint16_t(3))
        : "memory");
}

// ---------------------------------------------------------------- misc

__device__ __forceinline__ uint32_t elect_one_lane()
{
    return (threadIdx.x & 31) == 0;
}

// Named barriers take their id as an immediate, so ptxas reserves it for the kernel.
template <int ID, int NTHREADS>
__device__ __forceinline__ void named_barrier_sync()
{
    asm volatile("bar.sync %0, %1;" ::"n"(ID), "n"(NTHREADS) : "memory");
}

// Named barrier that also returns the OR of every participating thread's `pred` (one uniform decision).
template <int ID, int NTHREADS>
__device__ __forceinline__ bool named_barrier_or(bool pred)
{
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 q, %1, 0;\n\tbar.red.or.pred p, %2, %3, q;\n\tselp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(uint32_t(pred)), "n"(ID), "n"(NTHREADS)
        : "memory");
    return r != 0;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi)
{
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
}

}  // namespace mkb
