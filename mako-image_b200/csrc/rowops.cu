// Row and element kernels (see rowops.cuh).
#include "rowops.cuh"
#include "common.cuh"

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

// One warp per row; NV float4 per lane cover D = 128 * nv (nv <= NV).
template <int NV>
__global__ void __launch_bounds__(256) k_ln_mod(const LnModArgs a)
{
    const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    if (row >= a.rows)
        return;
    const int nv = a.D >> 7;
    const float4* xr = reinterpret_cast<const float4*>(a.x + long(row) * a.D);
    float4 v[NV];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv) {
            v[i] = xr[i * 32 + lane];
            s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        }
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
#pragma unroll
    for (int i = 0; i < NV; ++i)
        if (i < nv) {
            const int c = i * 32 + lane;
            const float4 g = __ldg(sc + c);
            float4 t = sh ? __ldg(sh + c) : make_float4(0.f, 0.f, 0.f, 0.f);
            yr[c] = pack4_bf16((v[i].x - mean) * rstd * (1.f + g.x) + t.x, (v[i].y - mean) * rstd * (1.f + g.y) + t.y,
                               (v[i].z - mean) * rstd * (1.f + g.z) + t.z, (v[i].w - mean) * rstd * (1.f + g.w) + t.w);
        }
}

template <int NV>
__global__ void __launch_bounds__(256) k_rms(const RmsArgs a)
{
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

// GEMV: x staged in shared memory; each warp takes 4 weight rows at a time, lanes stride the row in 16-byte chunks.
constexpr int kGemvRows = 4;

template <int B>
__global__ void __launch_bounds__(256) k_gemv(const __nv_bfloat16* __restrict__ W, const float* __restrict__ x,
                                              long ldx, const float* __restrict__ bias, float* __restrict__ y,
                                              long ldy, int N, int K, int act)
{
    extern __shared__ float xs[];  // [B][K]
    for (int i = threadIdx.x; i < B * K; i += blockDim.x)
        xs[i] = x[long(i / K) * ldx + i % K];
    __syncthreads();
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
                const float4 xa = *reinterpret_cast<const float4*>(xs + b * K + c * 8);
                const float4 xb = *reinterpret_cast<const float4*>(xs + b * K + c * 8 + 4);
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
    const int r = blockIdx.x, i = threadIdx.x;  // 128 threads
    if (r >= rows)
        return;
    const float freq = expf(-logf(10000.0f) * float(i) / 128.0f);
    const float arg = 1000.0f * t[r] * freq;
    tp[r * 256 + i] = cosf(arg);
    tp[r * 256 + 128 + i] = sinf(arg);
}

__device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void k_fill_normal(void* out, int bf16, uint64_t n, uint64_t key, uint64_t offset, float stdv, float mean)
{
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const uint64_t e = offset + i;
        const uint64_t h = splitmix64(key + (e >> 1));
        const double u1 = (double(h >> 40) + 0.5) / 16777216.0;
        const double u2 = double(h & 0xFFFFFFull) / 16777216.0;
        const double rr = sqrt(-2.0 * log(u1));
        const double ang = 6.283185307179586 * u2;
        const double z = (e & 1) ? rr * sin(ang) : rr * cos(ang);
        const float v = float(z * double(stdv) + double(mean));
        if (bf16)
            static_cast<__nv_bfloat16*>(out)[i] = __float2bfloat16_rn(v);
        else
            static_cast<float*>(out)[i] = v;
    }
}

__global__ void k_cast(const float* x, __nv_bfloat16* y, uint64_t n)
{
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = __float2bfloat16_rn(x[i]);
}

__global__ void k_silu(const float* x, float* y, uint64_t n)
{
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride)
        y[i] = x[i] / (1.0f + expf(-x[i]));
}

__global__ void k_copy_heads(const uint4* src, int src_rows, int src_off, uint4* dst, int dst_rows, int dst_off,
                             int heads, int rows)
{
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
    const uint64_t stride = uint64_t(gridDim.x) * blockDim.x;
    for (uint64_t i = uint64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += stride) {
        const float v = vu ? vu[i] + g * (vc[i] - vu[i]) : vc[i];
        x[i] += dt * v;
    }
}

int grid_for(uint64_t n, int threads)
{
    uint64_t g = (n + threads - 1) / threads;
    return int(g > 148ull * 32 ? 148ull * 32 : (g ? g : 1));
}

}  // namespace

cudaError_t ln_modulate(const LnModArgs& a, cudaStream_t st)
{
    if (a.D % 128 || a.D > 4096 || a.rows_per_sample <= 0)
        return cudaErrorInvalidValue;
    if (a.rows == 0)
        return cudaSuccess;
    const int nv = a.D / 128, blocks = (a.rows + 7) / 8;
    if (nv <= 8)
        k_ln_mod<8><<<blocks, 256, 0, st>>>(a);
    else if (nv <= 16)
        k_ln_mod<16><<<blocks, 256, 0, st>>>(a);
    else if (nv <= 24)
        k_ln_mod<24><<<blocks, 256, 0, st>>>(a);
    else
        k_ln_mod<32><<<blocks, 256, 0, st>>>(a);
    count_launch();
    return cudaGetLastError();
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
        k_rms<8><<<blocks, 256, 0, st>>>(a);
    else if (nv <= 16)
        k_rms<16><<<blocks, 256, 0, st>>>(a);
    else if (nv <= 24)
        k_rms<24><<<blocks, 256, 0, st>>>(a);
    else
        k_rms<32><<<blocks, 256, 0, st>>>(a);
    count_launch();
    return cudaGetLastError();
}

cudaError_t gemv(const __nv_bfloat16* W, const float* x, long ldx, const float* bias, float* y, long ldy, int B,
                 int N, int K, int act, cudaStream_t st)
{
    if (B < 1 || B > 8 || K % 8 || N <= 0 || (reinterpret_cast<uintptr_t>(W) & 15))
        return cudaErrorInvalidValue;
    const size_t smem = size_t(B) * K * sizeof(float);
    const int rows_per_block = 8 * kGemvRows;
    int blocks = (N + rows_per_block - 1) / rows_per_block;
    if (blocks > 148 * 8)
        blocks = 148 * 8;
    static size_t smem_set[9] = {};
#define MKB_GEMV(BB)                                                                                                   \
    case BB: {                                                                                                         \
        if (smem > 48 * 1024 && smem > smem_set[BB]) {                                                                 \
            cudaError_t e = cudaFuncSetAttribute(k_gemv<BB>, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)); \
            if (e != cudaSuccess)                                                                                      \
                return e;                                                                                              \
            smem_set[BB] = smem;                                                                                       \
        }                                                                                                              \
        k_gemv<BB><<<blocks, 256, smem, st>>>(W, x, ldx, bias, y, ldy, N, K, act);                                     \
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
    k_sinusoid<<<rows, 128, 0, st>>>(t, tp, rows);
    count_launch();
    return cudaGetLastError();
}

cudaError_t fill_normal(void* out, bool bf16, uint64_t n, uint64_t key, uint64_t offset, float std, float mean,
                        cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    k_fill_normal<<<grid_for(n, 256), 256, 0, st>>>(out, bf16 ? 1 : 0, n, key, offset, std, mean);
    count_launch();
    return cudaGetLastError();
}

cudaError_t cast_f32_bf16(const float* x, __nv_bfloat16* y, uint64_t n, cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    k_cast<<<grid_for(n, 256), 256, 0, st>>>(x, y, n);
    count_launch();
    return cudaGetLastError();
}

cudaError_t silu_f32(const float* x, float* y, uint64_t n, cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    k_silu<<<grid_for(n, 256), 256, 0, st>>>(x, y, n);
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
    k_copy_heads<<<grid_for(n, 256), 256, 0, st>>>(reinterpret_cast<const uint4*>(src), src_rows, src_off,
                                                   reinterpret_cast<uint4*>(dst), dst_rows, dst_off, heads, rows);
    count_launch();
    return cudaGetLastError();
}

cudaError_t cfg_euler(float* x, const float* v_c, const float* v_u, float g, float dt, uint64_t n, cudaStream_t st)
{
    if (!n)
        return cudaSuccess;
    k_cfg_euler<<<grid_for(n, 256), 256, 0, st>>>(x, v_c, v_u, g, dt, n);
    count_launch();
    return cudaGetLastError();
}

}  // namespace mkb
