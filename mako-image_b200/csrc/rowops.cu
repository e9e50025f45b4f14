// Row and element kernels (see rowops.cuh).
#include "rowops.cuh"
#include "common.cuh"
#include "launch.cuh"
#include "rng.cuh"

#include <algorithm>
#include <cstdint>

namespace mkb {

namespace {

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1)
        v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint2 pack4_bf16(float a, float b, float c, float d)
{
    __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
    return make_uint2(*reinterpret_cast<uint32_t*>(&lo), *reinterpret_cast<uint32_t*>(&hi));
}

// LayerNorm-modulate of one row by one warp: NV float4 per lane cover D = 128 * nv (nv <= NV).
template <int NV>
__device__ __forceinline__ void ln_load_row(const LnModArgs& a, int row, int lane, float4 (&v)[NV])
{
    const int nv = a.D >> 7;
    const float4* xr = reinterpret_cast<const float4*>(a.x + long(row) * a.D);
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv)
            v[i] = xr[i * 32 + lane];
}

template <int NV>
__device__ __forceinline__ void ln_finish_row(const LnModArgs& a, int row, int lane, const float4 (&v)[NV])
{
    const int nv = a.D >> 7;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv)
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    const float mean = warp_sum(s) / float(a.D);
    float q = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv) {
            const float dx = v[i].x - mean, dy = v[i].y - mean, dz = v[i].z - mean, dw = v[i].w - mean;
            q += (dx * dx + dy * dy) + (dz * dz + dw * dw);
        }
    const float rstd = rsqrtf(warp_sum(q) / float(a.D) + a.eps);
    const int sample = row / a.rows_per_sample, within = row - sample * a.rows_per_sample;
    const long moff = long(sample) * a.mod_stride + (within < a.split ? a.alt_off : 0);
    const float4* sc = reinterpret_cast<const float4*>(a.scale + moff);
    const float4* sh = a.shift ? reinterpret_cast<const float4*>(a.shift + moff) : nullptr;
    uint2* yr = reinterpret_cast<uint2*>(a.y + long(row) * a.D);
    const float off = a.affine ? 0.f : 1.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv) {
            const int c = i * 32 + lane;
            const float4 g = __ldg(sc + c);
            const float4 t = sh ? __ldg(sh + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            yr[c] = pack4_bf16((v[i].x - mean) * rstd * (off + g.x) + t.x, (v[i].y - mean) * rstd * (off + g.y) + t.y,
                               (v[i].z - mean) * rstd * (off + g.z) + t.z, (v[i].w - mean) * rstd * (off + g.w) + t.w);
        }
}

// The rows of up to two segments (same D), concatenated: global row g < rows0 is row g of s[0], else row g - rows0
// of s[1] (one launch for the text and image rows of a block).
struct LnSegs {
    LnModArgs s[2];
    int rows0, total;
};

// One warp per row: the grid's many independent row loads keep HBM busy (a persistent grid whose warps load their
// next row while normalising the current one measured 15-20% slower: half the rows in flight per SM).
template <int NV>
__global__ void __launch_bounds__(256) k_ln_mod(const __grid_constant__ LnSegs P)
{
    grid_dep_wait();
    grid_dep_launch();
    const int g = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (g >= P.total)
        return;
    const LnModArgs& a = g < P.rows0 ? P.s[0] : P.s[1];
    const int row = g < P.rows0 ? g : g - P.rows0;
    float4 v[NV];
    ln_load_row<NV>(a, row, lane, v);
    ln_finish_row<NV>(a, row, lane, v);
}

template <int NV>
__global__ void __launch_bounds__(256) k_rms(const RmsArgs a)
{
    grid_dep_wait();
    grid_dep_launch();
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= a.samples * a.rows_per_sample)
        return;
    const int nv = a.C >> 7;
    const int sample = row / a.rows_per_sample, within = row - sample * a.rows_per_sample;
    const float4* xr = reinterpret_cast<const float4*>(a.src[sample] + long(within) * a.C);
    float4 v[NV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv) {
            v[i] = xr[i * 32 + lane];
            s += (v[i].x * v[i].x + v[i].y * v[i].y) + (v[i].z * v[i].z + v[i].w * v[i].w);
        }
    const float r = rsqrtf(warp_sum(s) / float(a.C) + a.eps);
    const float4* w4 = reinterpret_cast<const float4*>(a.w);
    uint2* yr = reinterpret_cast<uint2*>(a.y + long(row) * a.C);
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv) {
            const int c = i * 32 + lane;
            const float4 g = __ldg(w4 + c);
            yr[c] = pack4_bf16(v[i].x * r * g.x, v[i].y * r * g.y, v[i].z * r * g.z, v[i].w * r * g.w);
        }
}

// GEMV: x staged in shared memory (XS) or read through L1 (no shared memory, so that its blocks fit beside a
// GEMM's on an SM); each warp takes 4 weight rows at a time, lanes stride the row in 16-byte chunks. Both forms do
// the same arithmetic in the same order.
constexpr int kGemvRows = 4;

template <int B, bool XS>
__global__ void __launch_bounds__(256) k_gemv(const __nv_bfloat16* __restrict__ W, const float* __restrict__ x,
                                              long ldx, const float* __restrict__ bias, float* __restrict__ y,
                                              long ldy, int N, int K, int act)
{
    grid_dep_wait();
    grid_dep_launch();
    extern __shared__ float xs[];  // [B][K]
    if constexpr (XS) {
        for (int i = threadIdx.x; i < B * K; i += blockDim.x)
            xs[i] = x[long(i / K) * ldx + i % K];
        __syncthreads();
    }
    const int lane = threadIdx.x & 31;
    const int warps = (gridDim.x * blockDim.x) >> 5;
    const int chunks = K >> 3;
    for (int n0 = ((blockIdx.x * blockDim.x + threadIdx.x) >> 5) * kGemvRows; n0 < N; n0 += warps * kGemvRows) {
        float acc[kGemvRows][B];
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b)
                acc[r][b] = 0.f;
        for (int c = lane; c < chunks; c += 32) {
            uint4 w[kGemvRows];
#pragma unroll
            for (int r = 0; r < kGemvRows; ++r)
                w[r] = n0 + r < N ? __ldg(reinterpret_cast<const uint4*>(W + long(n0 + r) * K) + c)
                                  : make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const float4 xa = XS ? *reinterpret_cast<const float4*>(xs + b * K + c * 8)
                                     : __ldg(reinterpret_cast<const float4*>(x + b * ldx + c * 8));
                const float4 xb = XS ? *reinterpret_cast<const float4*>(xs + b * K + c * 8 + 4)
                                     : __ldg(reinterpret_cast<const float4*>(x + b * ldx + c * 8 + 4));
#pragma unroll
                for (int r = 0; r < kGemvRows; ++r) {
                    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w[r]);
                    const float2 f0 = __bfloat1622float2(h[0]), f1 = __bfloat1622float2(h[1]);
                    const float2 f2 = __bfloat1622float2(h[2]), f3 = __bfloat1622float2(h[3]);
                    acc[r][b] += f0.x * xa.x + f0.y * xa.y + f1.x * xa.z + f1.y * xa.w + f2.x * xb.x + f2.y * xb.y +
                                 f3.x * xb.z + f3.y * xb.w;
                }
            }
        }
#pragma unroll
        for (int r = 0; r < kGemvRows; ++r)
#pragma unroll
            for (int b = 0; b < B; ++b) {
                float v = warp_sum(acc[r][b]);
                if (lane == 0 && n0 + r < N) {
                    if (bias)
                        v += bias[n0 + r];
                    if (act == 2)
                        v = v / (1.f + __expf(-v));
                    y[long(b) * ldy + n0 + r] = v;
                }
            }
    }
}

__global__ void k_sinusoid(const float* t, float* tp, int rows)
{
    grid_dep_wait();
    grid_dep_launch();
    const int r = blockIdx.x, i = threadIdx.x;  // 128 threads
    if (r >= rows)
        return;
    const float freq = expf(-logf(10000.0f) * float(i) / 128.0f);
    const float arg = 1000.0f * t[r] * freq;
    tp[r * 256 + i] = cosf(arg);
    tp[r * 256 + 128 + i] = sinf(arg);
}

__global__ void k_fill_normal(void* out, int bf16, uint64_t n, uint64_t key, uint64_t offset, float stdv, float mean)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const double z = counter_normal(key, offset + i);
        const float v = float(z * double(stdv) + double(mean));
        if (bf16)
            static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
        else
            static_cast<float*>(out)[i] = v;
    }
}

__global__ void k_cast_scalar(const float* x, __nv_bfloat16* y, uint64_t n)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = __float2bfloat16_rn(x[i]);
}

// fp32 -> bf16: float4 in, four bf16 out per step, four steps in flight; the n % 4 tail by scalars. Needs x 16-byte
// and y 8-byte aligned (k_cast_scalar otherwise).
__global__ void k_cast(const float* x, __nv_bfloat16* y, uint64_t n)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t n4 = n / 4, stride = uint64_t(gridDim.x) * blockDim.x;
    const float4* x4 = reinterpret_cast<const float4*>(x);
    uint2* y4 = reinterpret_cast<uint2*>(y);
    uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    for (; i + 3 * stride < n4; i += 4 * stride) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            v[u] = x4[i + u * stride];
#pragma unroll
        for (int u = 0; u < 4; ++u)
            y4[i + u * stride] = pack4_bf16(v[u].x, v[u].y, v[u].z, v[u].w);
    }
    for (; i < n4; i += stride) {
        const float4 v = x4[i];
        y4[i] = pack4_bf16(v.x, v.y, v.z, v.w);
    }
    for (uint64_t j = 4 * n4 + uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += stride)
        y[j] = __float2bfloat16_rn(x[j]);
}

__global__ void k_silu(const float* x, float* y, uint64_t n)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = x[i] / (1.0f + expf(-x[i]));
}

__global__ void k_copy_heads(const uint4* src, int src_rows, int src_off, uint4* dst, int dst_rows, int dst_off,
                             int heads, int rows)
{
    grid_dep_wait();
    grid_dep_launch();
    // 16 uint4 per 128-wide bf16 row
    const uint64_t total = uint64_t(heads) * rows * 16;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int c = int(i & 15);
        const uint64_t hr = i >> 4;
        const int r = int(hr % rows), h = int(hr / rows);
        dst[(uint64_t(h) * dst_rows + dst_off + r) * 16 + c] = src[(uint64_t(h) * src_rows + src_off + r) * 16 + c];
    }
}

__global__ void k_cfg_euler(float* x, const float* vc, const float* vu, float g, float dt, uint64_t n)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = vu ? vu[i] + g * (vc[i] - vu[i]) : vc[i];
        x[i] += dt * v;
    }
}

// ---- GroupNorm
//
// x is channels-last fp32 [B][HW][C]. Thread t of a 256-thread block owns channel quad q = t % Qb (Qb = min(C/4,
// 256); quads q + 256, q + 512, ... too when C > 1024) and pixel lane r = t / Qb of Rb = 256 / Qb lanes, so a warp
// reads contiguous float4s and no thread divides per element.

// Pixels per statistics chunk: about eight chunks per SM over the whole batch, at least 16 pixels (small images
// with many channels still spread over most SMs).
__host__ __device__ inline int gn_chunk_px(int B, int HW)
{
    const long want = (long(B) * HW + 8 * 148 - 1) / (8 * 148);
    return int(want < 16 ? 16 : want);
}

constexpr int kGnSegments = 32;  // segments per group of the statistics a convolution left (k_gn_finalize_parts)

// Chan et al.'s pairwise combination of (count, mean, M2).
__device__ __forceinline__ void chan_combine(float& n, float& mean, float& m2, float nb, float meanb, float m2b)
{
    const float nn = n + nb;
    if (nn <= 0.f)
        return;
    const float d = meanb - mean;
    mean += d * (nb / nn);
    m2 += m2b + d * d * (n * nb / nn);
    n = nn;
}

// Per (sample, chunk, group): count, mean and M2 of the chunk's pixels, from per-thread running (Welford)
// statistics per channel, combined through shared memory [Rb][C] by one thread per group.
__global__ void __launch_bounds__(256) k_gn_stats(const GnArgs a, int chunk_px, int nchunks)
{
    grid_dep_wait();
    grid_dep_launch();
    extern __shared__ float sh[];  // mean [Rb][C], M2 [Rb][C], count [Rb]
    const int chunk = blockIdx.x, b = blockIdx.y;
    const int Q = a.C / 4, Qb = Q < 256 ? Q : 256, Rb = 256 / Qb;
    const int t = threadIdx.x, r = t / Qb, q0 = t % Qb;
    const int p0 = chunk * chunk_px, np = min(chunk_px, a.HW - p0);
    float* smean = sh;
    float* sm2 = sh + Rb * a.C;
    float* scount = sh + 2 * Rb * a.C;
    if (r < Rb) {
        const float4* xb = reinterpret_cast<const float4*>(a.x + (long(b) * a.HW + p0) * a.C);
        float n = 0.f;
        for (int q = q0; q < Q; q += Qb) {
            float mean[4] = {0.f, 0.f, 0.f, 0.f}, m2[4] = {0.f, 0.f, 0.f, 0.f};
            n = 0.f;
            auto update = [&](const float4 v) {
                n += 1.f;
                const float rn = 1.f / n;
                const float xv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const float d = xv[k] - mean[k];
                    mean[k] += d * rn;
                    m2[k] += d * (xv[k] - mean[k]);
                }
            };
            // Four pixels' loads issued before their (serial) updates: four loads in flight per thread.
            int p = r;
            for (; p + 3 * Rb < np; p += 4 * Rb) {
                const float4 v0 = xb[long(p) * Q + q], v1 = xb[long(p + Rb) * Q + q];
                const float4 v2 = xb[long(p + 2 * Rb) * Q + q], v3 = xb[long(p + 3 * Rb) * Q + q];
                update(v0);
                update(v1);
                update(v2);
                update(v3);
            }
            for (; p < np; p += Rb)
                update(xb[long(p) * Q + q]);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                smean[r * a.C + 4 * q + k] = mean[k];
                sm2[r * a.C + 4 * q + k] = m2[k];
            }
        }
        if (q0 == 0)
            scount[r] = n;
    }
    __syncthreads();
    const int cpg = a.C / a.groups;
    for (int g = t; g < a.groups; g += blockDim.x) {
        float n = 0.f, mean = 0.f, m2 = 0.f;
        for (int rr = 0; rr < Rb; ++rr)
            for (int c = g * cpg; c < (g + 1) * cpg; ++c)
                chan_combine(n, mean, m2, scount[rr], smean[rr * a.C + c], sm2[rr * a.C + c]);
        float* o = a.ws + ((long(b) * nchunks + chunk) * a.groups + g) * 3;
        o[0] = n;
        o[1] = mean;
        o[2] = m2;
    }
}

// Per (sample, group): the chunks combined by a tree, then mean and 1 / sqrt(var + eps).
__global__ void __launch_bounds__(256) k_gn_finalize(const GnArgs a, int nchunks)
{
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float sn[256], sm[256], sq[256];
    const int g = blockIdx.x, b = blockIdx.y;
    float n = 0.f, mean = 0.f, m2 = 0.f;
    for (int k = threadIdx.x; k < nchunks; k += blockDim.x) {
        const float* o = a.ws + ((long(b) * nchunks + k) * a.groups + g) * 3;
        chan_combine(n, mean, m2, o[0], o[1], o[2]);
    }
    sn[threadIdx.x] = n;
    sm[threadIdx.x] = mean;
    sq[threadIdx.x] = m2;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            float nn = sn[threadIdx.x], mm = sm[threadIdx.x], qq = sq[threadIdx.x];
            chan_combine(nn, mm, qq, sn[threadIdx.x + w], sm[threadIdx.x + w], sq[threadIdx.x + w]);
            sn[threadIdx.x] = nn;
            sm[threadIdx.x] = mm;
            sq[threadIdx.x] = qq;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float* f = a.ws + long(a.B) * nchunks * a.groups * 3 + (long(b) * a.groups + g) * 2;
        f[0] = sm[0];
        f[1] = rsqrtf(sq[0] / fmaxf(sn[0], 1.f) + a.eps);
    }
}

// The statistics a convolution's epilogue left, float4 (count, mean, M2, 0) per [B][groups][nchunks] (a group's
// chunks contiguous, read coalesced), combined per segment of the chunks: block (g, b, s) writes segment s of group
// g as float4 (count, mean, M2, 0) at a.ws[((b * groups + g) * gridDim.z + s) * 4]. k_gn_apply combines the
// segments (a few per group) when it starts, so no single block walks all of a group's chunks.
__global__ void __launch_bounds__(256) k_gn_finalize_parts(const GnArgs a, const float4* parts, int nchunks)
{
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float sn[256], sm[256], sq[256];
    const int g = blockIdx.x, b = blockIdx.y, segs = gridDim.z;
    const int k0 = int(long(nchunks) * blockIdx.z / segs), k1 = int(long(nchunks) * (blockIdx.z + 1) / segs);
    const float4* p = parts + (long(b) * a.groups + g) * nchunks;
    float n = 0.f, mean = 0.f, m2 = 0.f;
    for (int k = k0 + threadIdx.x; k < k1; k += blockDim.x) {
        const float4 o = p[k];
        chan_combine(n, mean, m2, o.x, o.y, o.z);
    }
    sn[threadIdx.x] = n;
    sm[threadIdx.x] = mean;
    sq[threadIdx.x] = m2;
    __syncthreads();
    for (int w = blockDim.x / 2; w > 0; w >>= 1) {
        if (threadIdx.x < w) {
            float nn = sn[threadIdx.x], mm = sm[threadIdx.x], qq = sq[threadIdx.x];
            chan_combine(nn, mm, qq, sn[threadIdx.x + w], sm[threadIdx.x + w], sq[threadIdx.x + w]);
            sn[threadIdx.x] = nn;
            sm[threadIdx.x] = mm;
            sq[threadIdx.x] = qq;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0)
        reinterpret_cast<float4*>(a.ws)[(long(b) * a.groups + g) * segs + blockIdx.z] = make_float4(sn[0], sm[0], sq[0], 0.f);
}

// y = x * scale_c + shift_c (then SiLU) as bf16, scale_c = rstd_g gamma_c, shift_c = beta_c - mean_g scale_c; each
// thread keeps its quad's four (scale, shift) in registers. Block (x, b) covers pixels [x * px, (x + 1) * px).
// segs > 0: the statistics are k_gn_finalize_parts' segments, combined here per group into shared memory first.
__global__ void __launch_bounds__(256) k_gn_apply(const GnArgs a, int nchunks, int px, int segs)
{
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float sfin[2 * 256];
    const int b = blockIdx.y;
    const float* fin = a.ws + long(a.B) * nchunks * a.groups * 3 + long(b) * a.groups * 2;
    if (segs > 0) {
        // Eight lanes per group, each combining every eighth segment, then the lanes' results by shuffles.
        for (int base = 0; base < a.groups * 8; base += blockDim.x) {
            const int idx = base + threadIdx.x, g = idx >> 3, l = idx & 7;
            float n = 0.f, mean = 0.f, m2 = 0.f;
            if (g < a.groups) {
                const float4* s = reinterpret_cast<const float4*>(a.ws) + (long(b) * a.groups + g) * segs;
                for (int k = l; k < segs; k += 8) {
                    const float4 o = s[k];
                    chan_combine(n, mean, m2, o.x, o.y, o.z);
                }
            }
#pragma unroll
            for (int off = 4; off > 0; off >>= 1) {
                const float n2 = __shfl_xor_sync(0xffffffffu, n, off), mean2 = __shfl_xor_sync(0xffffffffu, mean, off),
                            m22 = __shfl_xor_sync(0xffffffffu, m2, off);
                chan_combine(n, mean, m2, n2, mean2, m22);
            }
            if (g < a.groups && l == 0) {
                sfin[2 * g] = mean;
                sfin[2 * g + 1] = rsqrtf(m2 / fmaxf(n, 1.f) + a.eps);
            }
        }
        __syncthreads();
        fin = sfin;
    }
    const int Q = a.C / 4, Qb = Q < 256 ? Q : 256, Rb = 256 / Qb;
    const int t = threadIdx.x, r = t / Qb, q0 = t % Qb;
    if (r >= Rb)
        return;
    const int p0 = blockIdx.x * px, np = min(px, a.HW - p0);
    const int cpg = a.C / a.groups;
    const float4* xb = reinterpret_cast<const float4*>(a.x + (long(b) * a.HW + p0) * a.C);
    uint2* yb = reinterpret_cast<uint2*>(a.y + (long(b) * a.HW + p0) * a.C);
    for (int q = q0; q < Q; q += Qb) {
        float sc[4], sf[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const int c = 4 * q + k, g = c / cpg;
            sc[k] = fin[2 * g + 1] * a.gamma[c];
            sf[k] = (a.beta ? a.beta[c] : 0.f) - fin[2 * g] * sc[k];
        }
        int p = r;
        for (; p + 3 * Rb < np; p += 4 * Rb) {  // four loads in flight
            float4 v[4];
#pragma unroll
            for (int u = 0; u < 4; ++u)
                v[u] = xb[long(p + u * Rb) * Q + q];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                float y[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    y[k] = fmaf(y[k], sc[k], sf[k]);
                    if (a.silu)
                        y[k] = y[k] / (1.f + __expf(-y[k]));
                }
                yb[long(p + u * Rb) * Q + q] = pack4_bf16(y[0], y[1], y[2], y[3]);
            }
        }
        for (; p < np; p += Rb) {
            const float4 v = xb[long(p) * Q + q];
            float y[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                y[k] = fmaf(y[k], sc[k], sf[k]);
                if (a.silu)
                    y[k] = y[k] / (1.f + __expf(-y[k]));
            }
            yb[long(p) * Q + q] = pack4_bf16(y[0], y[1], y[2], y[3]);
        }
    }
}

// Nearest 2x upsampling: block (y, b) reads input row y once (float4 per thread, the quad/lane mapping of the
// GroupNorm kernels) and writes it to output rows 2y and 2y + 1, each pixel twice.
__global__ void __launch_bounds__(256) k_upsample2x(const float4* x, uint2* y, int H, int W, int Q)
{
    grid_dep_wait();
    grid_dep_launch();
    const int iy = blockIdx.x, b = blockIdx.y;
    const int Qb = Q < 256 ? Q : 256, Rb = 256 / Qb;
    const int t = threadIdx.x, r = t / Qb, q0 = t % Qb;
    if (r >= Rb)
        return;
    const float4* xr = x + (long(b) * H + iy) * W * Q;
    uint2* y0 = y + (long(b) * 2 * H + 2 * iy) * 2 * W * Q;
    uint2* y1 = y0 + long(2 * W) * Q;
    for (int q = q0; q < Q; q += Qb)
        for (int ix = r; ix < W; ix += Rb) {
            const float4 v = xr[long(ix) * Q + q];
            const uint2 o = pack4_bf16(v.x, v.y, v.z, v.w);
            const long j = long(2 * ix) * Q + q;
            y0[j] = o;
            y0[j + Q] = o;
            y1[j] = o;
            y1[j + Q] = o;
        }
}

__global__ void k_concat(const float4* a, int Ca4, const float4* b, int Cb4, float4* y, long P)
{
    grid_dep_wait();
    grid_dep_launch();
    const int C4 = Ca4 + Cb4;
    const uint64_t total = uint64_t(P) * C4;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int c = int(i % C4);
        const uint64_t p = i / C4;
        y[i] = c < Ca4 ? a[p * Ca4 + c] : b[p * Cb4 + (c - Ca4)];
    }
}

__global__ void k_pad_channels(const float* x, int C, __nv_bfloat16* y, int Cp, long P)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t total = uint64_t(P) * Cp;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int c = int(i % Cp);
        const uint64_t p = i / Cp;
        y[i] = __float2bfloat16_rn(c < C ? x[p * C + c] : 0.f);
    }
}

__global__ void k_unpack(const float* tok, __nv_bfloat16* img, int B, int gh, int gw, int Cp, float scale)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t total = uint64_t(B) * 4 * gh * gw * Cp;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int c = int(i % Cp);
        const uint64_t px = i / Cp;
        const int x = int(px % (2 * gw)), y = int((px / (2 * gw)) % (2 * gh)), b = int(px / (4ull * gh * gw));
        float v = 0.f;
        if (c < 4)
            v = tok[((uint64_t(b) * gh + y / 2) * gw + x / 2) * 16 + c * 4 + (y % 2) * 2 + x % 2] * scale;
        img[i] = __float2bfloat16_rn(v);
    }
}

// Tokens [gh*gw][4 z] of one image to its channels-last latent image [2gh][2gw][Cp] bf16: token value
// i = (c * 2 + py) * 2 + px is channel c of pixel (2y + py, 2x + px), mapped to v * aff[i] + aff[4 z + i] (the
// VAE's per-value latent statistics); channels z..Cp-1 are zero.
__global__ void k_unpack_affine(const float* tok, __nv_bfloat16* img, int gh, int gw, int z, int Cp, const float* aff)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t total = uint64_t(4) * gh * gw * Cp;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int c = int(i % Cp);
        const uint64_t px = i / Cp;
        const int x = int(px % (2 * gw)), y = int(px / (2 * gw));
        float v = 0.f;
        if (c < z) {
            const int k = c * 4 + (y % 2) * 2 + x % 2;
            v = tok[(uint64_t(y / 2) * gw + x / 2) * 4 * z + k] * aff[k] + aff[4 * z + k];
        }
        img[i] = __float2bfloat16_rn(v);
    }
}

__global__ void k_pack(const float* img, int Cs, float* tok, int B, int gh, int gw)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t total = uint64_t(B) * gh * gw * 16;
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
        const int j = int(i % 16);
        const uint64_t t = i / 16;
        const int tx = int(t % gw), ty = int((t / gw) % gh), b = int(t / (uint64_t(gh) * gw));
        const int c = j / 4, y = 2 * ty + (j % 4) / 2, x = 2 * tx + j % 2;
        tok[i] = img[((uint64_t(b) * 2 * gh + y) * 2 * gw + x) * Cs + c];
    }
}

__global__ void k_add_silu(const float* a, const float* b, float* out, uint64_t n)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = a[i] + b[i];
        out[i] = v / (1.f + expf(-v));
    }
}

__global__ void k_to_rgba(const float* img, int Cs, float4* rgba, long P)
{
    grid_dep_wait();
    grid_dep_launch();
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t p = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; p < uint64_t(P); p += stride) {
        const float* s = img + p * Cs;
        rgba[p] = make_float4(fminf(fmaxf(s[0], -1.f), 1.f), fminf(fmaxf(s[1], -1.f), 1.f),
                              fminf(fmaxf(s[2], -1.f), 1.f), 1.f);
    }
}

// One CTA per row: max, then exp-sum, then normalised bf16 probabilities.
__global__ void __launch_bounds__(256) k_softmax_rows(const float* s, __nv_bfloat16* p, int n, float scale)
{
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float red[32];
    const float* r = s + long(blockIdx.x) * n;
    __nv_bfloat16* o = p + long(blockIdx.x) * n;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        m = fmaxf(m, r[i] * scale);
    for (int k = 16; k; k >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, k));
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < blockDim.x / 32; ++w)
        m = fmaxf(m, red[w]);
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        sum += __expf(r[i] * scale - m);
    sum = warp_sum(sum);
    if ((threadIdx.x & 31) == 0)
        red[threadIdx.x >> 5] = sum;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < blockDim.x / 32; ++w)
        tot += red[w];
    const float inv = 1.f / tot;
    for (int i = threadIdx.x; i < n; i += blockDim.x)
        o[i] = __float2bfloat16_rn(__expf(r[i] * scale - m) * inv);
}

// The same softmax with the row held in shared memory (n * 4 bytes, 512 threads): one read of s instead of three.
// The scaled scores, then their exponentials, stay in shared memory between the passes.
__global__ void __launch_bounds__(512) k_softmax_rows_smem(const float* s, __nv_bfloat16* p, int n, float scale)
{
    grid_dep_wait();
    grid_dep_launch();
    extern __shared__ float4 srow[];
    __shared__ float red[16];
    const float4* r = reinterpret_cast<const float4*>(s + long(blockIdx.x) * n);
    const int n4 = n / 4, warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 v = r[i];
        v.x *= scale;
        v.y *= scale;
        v.z *= scale;
        v.w *= scale;
        srow[i] = v;
        m = fmaxf(m, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
    }
    for (int k = 16; k; k >>= 1)
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, k));
    if (lane == 0)
        red[warp] = m;
    __syncthreads();
    m = red[0];
    for (int w = 1; w < blockDim.x / 32; ++w)
        m = fmaxf(m, red[w]);
    __syncthreads();
    float sum = 0.f;
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        float4 v = srow[i];
        v.x = __expf(v.x - m);
        v.y = __expf(v.y - m);
        v.z = __expf(v.z - m);
        v.w = __expf(v.w - m);
        srow[i] = v;
        sum += (v.x + v.y) + (v.z + v.w);
    }
    sum = warp_sum(sum);
    if (lane == 0)
        red[warp] = sum;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < blockDim.x / 32; ++w)
        tot += red[w];
    const float inv = 1.f / tot;
    uint2* o = reinterpret_cast<uint2*>(p + long(blockIdx.x) * n);
    for (int i = threadIdx.x; i < n4; i += blockDim.x) {
        const float4 v = srow[i];
        o[i] = pack4_bf16(v.x * inv, v.y * inv, v.z * inv, v.w * inv);
    }
}

__global__ void k_transpose(const __nv_bfloat16* x, long ldx, int c0, __nv_bfloat16* y, long rows, int cols)
{
    grid_dep_wait();
    grid_dep_launch();
    __shared__ __nv_bfloat16 tile[32][33];
    const long r0 = long(blockIdx.x) * 32;
    const int cb = blockIdx.y * 32;
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const long r = r0 + k;
        const int c = cb + threadIdx.x;
        if (r < rows && c < cols)
            tile[k][threadIdx.x] = x[r * ldx + c0 + c];
    }
    __syncthreads();
    for (int k = threadIdx.y; k < 32; k += blockDim.y) {
        const int c = cb + k;
        const long r = r0 + threadIdx.x;
        if (r < rows && c < cols)
            y[long(c) * rows + r] = tile[threadIdx.x][k];
    }
}

// ---------------------------------------------------------------- SDXL text encoders (sdxl.cpp:459-546)

// x[m][e] = tok[ids[m]][e] + pos[m % T][e]: a token's embedding row plus its position's. One block per row.
__global__ void __launch_bounds__(256) k_clip_embed(const int* ids, const float* tok, const float* pos, float* x,
                                                   int T, int E)
{
    grid_dep_wait();
    grid_dep_launch();
    const int m = blockIdx.x;
    const float* t = tok + long(ids[m]) * E;
    const float* p = pos + long(m % T) * E;
    float* y = x + long(m) * E;
    for (int e = threadIdx.x; e < E; e += blockDim.x)
        y[e] = t[e] + p[e];
}

// The bf16 rounding of v and of what it left out, packed as y[col] and y[N + col] of a row of 2N.
__device__ __forceinline__ void split_store(__nv_bfloat16* y, int N, int col, float v)
{
    const __nv_bfloat16 hi = __float2bfloat16_rn(v);
    y[col] = hi;
    y[N + col] = __float2bfloat16_rn(v - __bfloat162float(hi));
}

// LayerNorm of fp32 rows (two passes over the row for mean and variance), the result split into bf16 parts. One
// warp per row.
__global__ void __launch_bounds__(256) k_ln_split(const float* x, const float* g, const float* b, __nv_bfloat16* y,
                                                 int M, int E, float eps)
{
    grid_dep_wait();
    grid_dep_launch();
    const int m = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x % 32;
    if (m >= M)
        return;
    const float* r = x + long(m) * E;
    float s = 0.f;
    for (int e = lane; e < E; e += 32)
        s += r[e];
    const float mean = warp_sum(s) / E;
    float q = 0.f;
    for (int e = lane; e < E; e += 32) {
        const float d = r[e] - mean;
        q = fmaf(d, d, q);
    }
    const float inv = rsqrtf(warp_sum(q) / E + eps);
    __nv_bfloat16* o = y + long(m) * 2 * E;
    for (int e = lane; e < E; e += 32)
        split_store(o, E, e, (r[e] - mean) * inv * g[e] + b[e]);
}

__global__ void __launch_bounds__(256) k_split_bf16(const float* x, __nv_bfloat16* y, long M, int N)
{
    grid_dep_wait();
    grid_dep_launch();
    const long n = M * N;
    for (long i = blockIdx.x * long(blockDim.x) + threadIdx.x; i < n; i += long(gridDim.x) * blockDim.x) {
        const long m = i / N;
        split_store(y + m * 2 * N, N, int(i - m * N), x[i]);
    }
}

// bigG's pooled state per chunk b: LayerNorm of row eos[b] of chunk b, times proj [E][P] as stored. One block per
// chunk; the normed row in shared memory, each thread a strided set of output columns (coalesced proj rows).
__global__ void __launch_bounds__(256) k_clip_pooled(const float* x, const int* eos, const float* g, const float* b,
                                                    const float* proj, float* out, int T, int E, int P, float eps)
{
    grid_dep_wait();
    grid_dep_launch();
    __shared__ float row[2048];
    __shared__ float red[8];
    const int c = blockIdx.x, t = threadIdx.x;
    const float* r = x + (long(c) * T + eos[c]) * E;
    auto block_sum = [&](float v) {
        v = warp_sum(v);
        if (t % 32 == 0)
            red[t / 32] = v;
        __syncthreads();
        float s = 0.f;
        for (int w = 0; w < 8; ++w)
            s += red[w];
        __syncthreads();
        return s;
    };
    float s = 0.f;
    for (int e = t; e < E; e += 256) {
        row[e] = r[e];
        s += row[e];
    }
    const float mean = block_sum(s) / E;
    float q = 0.f;
    for (int e = t; e < E; e += 256) {
        const float d = row[e] - mean;
        q = fmaf(d, d, q);
    }
    const float inv = rsqrtf(block_sum(q) / E + eps);
    for (int e = t; e < E; e += 256)
        row[e] = (row[e] - mean) * inv * g[e] + b[e];
    __syncthreads();
    for (int j = t; j < P; j += 256) {
        float acc = 0.f;
        for (int i = 0; i < E; ++i)
            acc = fmaf(row[i], proj[long(i) * P + j], acc);
        out[long(c) * P + j] = acc;
    }
}

int grid_for(uint64_t n, int threads)
{
    uint64_t g = (n + threads - 1) / threads;
    return int(g > 148ull * 32 ? 148ull * 32 : (g ? g : 1));
}

}  // namespace

namespace {

bool ln_args_ok(const LnModArgs& a) { return a.D % 128 == 0 && a.D <= 4096 && a.rows_per_sample > 0 && a.rows >= 0; }

}  // namespace

cudaError_t ln_modulate2(const LnModArgs& a, const LnModArgs& b, cudaStream_t st)
{
    if (!ln_args_ok(a) || !ln_args_ok(b) || (a.rows && b.rows && a.D != b.D))
        return cudaErrorInvalidValue;
    LnSegs P;
    P.s[0] = a;
    P.s[1] = b;
    P.rows0 = a.rows;
    P.total = a.rows + b.rows;
    if (P.total == 0)
        return cudaSuccess;
    const int nv = (a.rows ? a.D : b.D) / 128, blocks = (P.total + 7) / 8;
    if (nv <= 8)
        launch_k(k_ln_mod<8>, blocks, 256, 0, st, P);
    else if (nv <= 16)
        launch_k(k_ln_mod<16>, blocks, 256, 0, st, P);
    else if (nv <= 24)
        launch_k(k_ln_mod<24>, blocks, 256, 0, st, P);
    else
        launch_k(k_ln_mod<32>, blocks, 256, 0, st, P);
    count_launch();
    return cudaGetLastError();
}

cudaError_t ln_modulate(const LnModArgs& a, cudaStream_t st)
{
    LnModArgs none = a;
    none.rows = 0;
    return ln_modulate2(a, none, st);
}

cudaError_t rms_norm_rows(const RmsArgs& a, cudaStream_t st)
{
    if (a.C % 128 || a.C > 4096 || a.samples <= 0 || a.samples > 8)
        return cudaErrorInvalidValue;
    const int rows = a.samples * a.rows_per_sample;
    if (rows == 0)
        return cudaSuccess;
    const int nv = a.C / 128, blocks = (rows + 7) / 8;
    if (nv <= 8)
        launch_k(k_rms<8>, blocks, 256, 0, st, a);
    else if (nv <= 16)
        launch_k(k_rms<16>, blocks, 256, 0, st, a);
    else if (nv <= 24)
        launch_k(k_rms<24>, blocks, 256, 0, st, a);
    else
        launch_k(k_rms<32>, blocks, 256, 0, st, a);
    count_launch();
    return cudaGetLastError();
}

cudaError_t gemv(const __nv_bfloat16* W, const float* x, long ldx, const float* bias, float* y, long ldy, int B,
                 int N, int K, int act, cudaStream_t st, bool no_smem)
{
    if (B < 1 || B > 8 || K % 8 || N <= 0 || (reinterpret_cast<uintptr_t>(W) & 15) ||
        (no_smem && ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx & 3))))
        return cudaErrorInvalidValue;
    const size_t smem = no_smem ? 0 : size_t(B) * K * sizeof(float);
    const int rows_per_block = 8 * kGemvRows;
    int blocks = (N + rows_per_block - 1) / rows_per_block;
    if (blocks > 148 * 8)
        blocks = 148 * 8;
    // Above 48 KB the limit is raised on every such launch: it belongs to the current device, and the sizes vary.
#define MKB_GEMV(BB)                                                                                                   \
    case BB: {                                                                                                         \
        if (no_smem) {                                                                                                 \
            launch_k(k_gemv<BB, false>, blocks, 256, 0, st, W, x, ldx, bias, y, ldy, N, K, act);                       \
            break;                                                                                                     \
        }                                                                                                              \
        if (smem > 48 * 1024) {                                                                                        \
            cudaError_t e =                                                                                            \
                cudaFuncSetAttribute(k_gemv<BB, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));       \
            if (e != cudaSuccess)                                                                                      \
                return e;                                                                                              \
        }                                                                                                              \
        launch_k(k_gemv<BB, true>, blocks, 256, smem, st, W, x, ldx, bias, y, ldy, N, K, act);                         \
        break;                                                                                                         \
    }
    switch (B) {
        MKB_GEMV(1)
        MKB_GEMV(2)
        MKB_GEMV(3)
        MKB_GEMV(4)
        MKB_GEMV(5)
        MKB_GEMV(6)
        MKB_GEMV(7)
        MKB_GEMV(8)
    }
#undef MKB_GEMV
    count_launch();
    return cudaGetLastError();
}

cudaError_t timestep_sinusoid(const float* t, float* tp, int rows, cudaStream_t st)
{
    if (rows <= 0)
        return cudaSuccess;
    launch_k(k_sinusoid, rows, 128, 0, st, t, tp, rows);
    count_launch();
    return cudaGetLastError();
}

cudaError_t fill_normal(void* out, bool bf16, uint64_t n, uint64_t key, uint64_t offset, float std, float mean,
                        cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    launch_k(k_fill_normal, grid_for(n, 256), 256, 0, st, out, bf16 ? 1 : 0, n, key, offset, std, mean);
    count_launch();
    return cudaGetLastError();
}

cudaError_t cast_f32_bf16(const float* x, __nv_bfloat16* y, uint64_t n, cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(y) & 7))
        launch_k(k_cast_scalar, grid_for(n, 256), 256, 0, st, x, y, n);
    else
        launch_k(k_cast, grid_for(n / 4 + 1, 256), 256, 0, st, x, y, n);
    count_launch();
    return cudaGetLastError();
}

cudaError_t silu_f32(const float* x, float* y, uint64_t n, cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    launch_k(k_silu, grid_for(n, 256), 256, 0, st, x, y, n);
    count_launch();
    return cudaGetLastError();
}

cudaError_t copy_head_rows(const __nv_bfloat16* src, int src_rows, int src_off, __nv_bfloat16* dst, int dst_rows,
                           int dst_off, int heads, int rows, cudaStream_t st)
{
    if (rows <= 0 || heads <= 0)
        return cudaSuccess;
    if (src_off + rows > src_rows || dst_off + rows > dst_rows)
        return cudaErrorInvalidValue;
    const uint64_t n = uint64_t(heads) * rows * 16;
    launch_k(k_copy_heads, grid_for(n, 256), 256, 0, st, reinterpret_cast<const uint4*>(src), src_rows, src_off,
             reinterpret_cast<uint4*>(dst), dst_rows, dst_off, heads, rows);
    count_launch();
    return cudaGetLastError();
}

size_t group_norm_workspace(int B, int HW, int C, int groups)
{
    (void)C;
    const size_t px = gn_chunk_px(B, HW), nchunks = (size_t(HW) + px - 1) / px;
    return (size_t(B) * nchunks * groups * 3 + size_t(B) * groups * 2) * sizeof(float);
}

cudaError_t group_norm(const GnArgs& a, cudaStream_t st)
{
    if (a.B <= 0 || a.HW <= 0 || a.groups <= 0 || a.C % a.groups || a.C % 4 || a.C > 6144 || !a.ws || !a.gamma)
        return cudaErrorInvalidValue;
    const int px = gn_chunk_px(a.B, a.HW), nchunks = (a.HW + px - 1) / px;
    const int Q = a.C / 4, Rb = 256 / (Q < 256 ? Q : 256);
    const size_t smem = (size_t(2) * Rb * a.C + Rb) * sizeof(float);  // <= 48 KB + 4 B at C = 6144
    static std::atomic<uint64_t> attr_devs{0};
    const cudaError_t e = smem_limit_once(attr_devs, k_gn_stats, (2 * 6144 + 1) * int(sizeof(float)));
    if (e != cudaSuccess)
        return e;
    launch_k(k_gn_stats, dim3(nchunks, a.B), 256, smem, st, a, px, nchunks);
    count_launch();
    launch_k(k_gn_finalize, dim3(a.groups, a.B), 256, 0, st, a, nchunks);
    count_launch();
    // Apply: about eight blocks per SM over the batch.
    const int apx = int(std::max<long>(16, (long(a.B) * a.HW + 8 * 148 - 1) / (8 * 148)));
    launch_k(k_gn_apply, dim3((a.HW + apx - 1) / apx, a.B), 256, 0, st, a, nchunks, apx, 0);
    count_launch();
    return cudaGetLastError();
}

cudaError_t group_norm_from_parts(const GnArgs& a, const float4* parts, int nchunks, cudaStream_t st)
{
    if (a.B <= 0 || a.HW <= 0 || a.groups <= 0 || a.groups > 256 || a.C % a.groups || a.C % 4 || !a.ws ||
        (reinterpret_cast<uintptr_t>(a.ws) & 15) || !a.gamma || !parts || nchunks <= 0)
        return cudaErrorInvalidValue;
    const int segs = std::min(kGnSegments, nchunks);
    launch_k(k_gn_finalize_parts, dim3(a.groups, a.B, segs), 256, 0, st, a, parts, nchunks);
    count_launch();
    const int apx = int(std::max<long>(16, (long(a.B) * a.HW + 8 * 148 - 1) / (8 * 148)));
    launch_k(k_gn_apply, dim3((a.HW + apx - 1) / apx, a.B), 256, 0, st, a, 0, apx, segs);
    count_launch();
    return cudaGetLastError();
}

cudaError_t upsample2x_bf16(const float* x, __nv_bfloat16* y, int B, int H, int W, int C, cudaStream_t st)
{
    if (C % 4 || B <= 0 || H <= 0 || W <= 0)
        return cudaErrorInvalidValue;
    launch_k(k_upsample2x, dim3(H, B), 256, 0, st, reinterpret_cast<const float4*>(x), reinterpret_cast<uint2*>(y),
             H, W, C / 4);
    count_launch();
    return cudaGetLastError();
}

cudaError_t concat_channels(const float* a, int Ca, const float* b, int Cb, float* y, long P, cudaStream_t st)
{
    if (Ca % 4 || Cb % 4)
        return cudaErrorInvalidValue;
    const uint64_t n = uint64_t(P) * (Ca + Cb) / 4;
    launch_k(k_concat, grid_for(n, 256), 256, 0, st, reinterpret_cast<const float4*>(a), Ca / 4,
             reinterpret_cast<const float4*>(b), Cb / 4, reinterpret_cast<float4*>(y), P);
    count_launch();
    return cudaGetLastError();
}

cudaError_t pad_channels_bf16(const float* x, int C, __nv_bfloat16* y, int Cp, long P, cudaStream_t st)
{
    if (C > Cp)
        return cudaErrorInvalidValue;
    const uint64_t n = uint64_t(P) * Cp;
    launch_k(k_pad_channels, grid_for(n, 256), 256, 0, st, x, C, y, Cp, P);
    count_launch();
    return cudaGetLastError();
}

cudaError_t unpack_tokens_bf16(const float* tokens, __nv_bfloat16* img, int B, int gh, int gw, int Cp, float scale,
                               cudaStream_t st)
{
    const uint64_t n = uint64_t(B) * 4 * gh * gw * Cp;
    launch_k(k_unpack, grid_for(n, 256), 256, 0, st, tokens, img, B, gh, gw, Cp, scale);
    count_launch();
    return cudaGetLastError();
}

cudaError_t unpack_tokens_affine_bf16(const float* tokens, __nv_bfloat16* img, int gh, int gw, int z, int Cp,
                                      const float* affine, cudaStream_t st)
{
    if (z < 1 || z > Cp)
        return cudaErrorInvalidValue;
    const uint64_t n = uint64_t(4) * gh * gw * Cp;
    launch_k(k_unpack_affine, grid_for(n, 256), 256, 0, st, tokens, img, gh, gw, z, Cp, affine);
    count_launch();
    return cudaGetLastError();
}

cudaError_t pack_tokens(const float* img, int Cs, float* tokens, int B, int gh, int gw, cudaStream_t st)
{
    const uint64_t n = uint64_t(B) * gh * gw * 16;
    launch_k(k_pack, grid_for(n, 256), 256, 0, st, img, Cs, tokens, B, gh, gw);
    count_launch();
    return cudaGetLastError();
}

cudaError_t add_silu(const float* a, const float* b, float* out, uint64_t n, cudaStream_t st)
{
    launch_k(k_add_silu, grid_for(n, 256), 256, 0, st, a, b, out, n);
    count_launch();
    return cudaGetLastError();
}

cudaError_t to_rgba(const float* img, int Cs, float* rgba, long P, cudaStream_t st)
{
    launch_k(k_to_rgba, grid_for(P, 256), 256, 0, st, img, Cs, reinterpret_cast<float4*>(rgba), P);
    count_launch();
    return cudaGetLastError();
}

cudaError_t softmax_rows_bf16(const float* s, __nv_bfloat16* p, long rows, int n, float scale, cudaStream_t st)
{
    // Rows of up to 24K floats (96 KB: two or more blocks per SM) are held in shared memory.
    const size_t smem = size_t(n) * 4;
    if (n % 4 == 0 && smem <= 96 * 1024 && !(reinterpret_cast<uintptr_t>(s) & 15) &&
        !(reinterpret_cast<uintptr_t>(p) & 7)) {
        static std::atomic<uint64_t> attr_devs{0};
        if (smem > 48 * 1024) {
            const cudaError_t e = smem_limit_once(attr_devs, k_softmax_rows_smem, 96 * 1024);
            if (e != cudaSuccess)
                return e;
        }
        launch_k(k_softmax_rows_smem, dim3(unsigned(rows)), 512, smem, st, s, p, n, scale);
        count_launch();
        return cudaGetLastError();
    }
    launch_k(k_softmax_rows, dim3(unsigned(rows)), 256, 0, st, s, p, n, scale);
    count_launch();
    return cudaGetLastError();
}

cudaError_t transpose_bf16(const __nv_bfloat16* x, long ldx, int c0, __nv_bfloat16* y, long rows, int cols,
                           cudaStream_t st)
{
    dim3 grid(unsigned((rows + 31) / 32), unsigned((cols + 31) / 32));
    launch_k(k_transpose, grid, dim3(32, 8), 0, st, x, ldx, c0, y, rows, cols);
    count_launch();
    return cudaGetLastError();
}

cudaError_t clip_embed(const int* ids, const float* tok, const float* pos, float* x, int M, int T, int E,
                       cudaStream_t st)
{
    if (M <= 0 || T <= 0 || E <= 0)
        return cudaErrorInvalidValue;
    launch_k(k_clip_embed, dim3(M), 256, 0, st, ids, tok, pos, x, T, E);
    count_launch();
    return cudaGetLastError();
}

cudaError_t ln_split_bf16(const float* x, const float* g, const float* b, __nv_bfloat16* y, int M, int E, float eps,
                          cudaStream_t st)
{
    if (M <= 0 || E <= 0)
        return cudaErrorInvalidValue;
    launch_k(k_ln_split, dim3((M + 7) / 8), 256, 0, st, x, g, b, y, M, E, eps);
    count_launch();
    return cudaGetLastError();
}

cudaError_t split_bf16(const float* x, __nv_bfloat16* y, long M, int N, cudaStream_t st)
{
    if (M <= 0 || N <= 0)
        return cudaErrorInvalidValue;
    launch_k(k_split_bf16, grid_for(uint64_t(M) * N, 256), 256, 0, st, x, y, M, N);
    count_launch();
    return cudaGetLastError();
}

cudaError_t clip_pooled(const float* x, const int* eos, const float* g, const float* b, const float* proj, float* out,
                        int B, int T, int E, int P, float eps, cudaStream_t st)
{
    if (B <= 0 || E <= 0 || E > 2048 || P <= 0)
        return cudaErrorInvalidValue;
    launch_k(k_clip_pooled, dim3(B), 256, 0, st, x, eos, g, b, proj, out, T, E, P, eps);
    count_launch();
    return cudaGetLastError();
}

cudaError_t cfg_euler(float* x, const float* v_c, const float* v_u, float g, float dt, uint64_t n, cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    launch_k(k_cfg_euler, grid_for(n, 256), 256, 0, st, x, v_c, v_u, g, dt, n);
    count_launch();
    return cudaGetLastError();
}

}  // namespace mkb
