// Sampler updates on device latents (include/mkb_image.h, "Samplers on the device"): the guided combination, the
// Euler-ancestral step and the ER-SDE step of Engine::generate's loop (src/image/engine.cpp:471-506), so a denoising
// run keeps its latents on the GPU. The scalars (ancestral split, ER-SDE coefficients) are computed on the host in
// double precision exactly as the reference computes them; the kernels apply them per element with the reference's
// float / double mix. Noise comes from the counter-based generator (rng.cuh): element j of a step draws element
// (offset + j) of the stream `key`, so runs are reproducible and the oracle draws the same numbers.
#include "../host/er_sde_coef.hpp"
#include "common.cuh"
#include "launch.cuh"
#include "rng.cuh"

#include <algorithm>
#include <cmath>

namespace mkb {

namespace {

int grid_of(long n) { return int(std::min<long>((n + 255) / 256, 148L * 16)); }

__global__ void k_axpy(float* x, const float* v, float a, long n)
{
    grid_dep_wait();
    grid_dep_launch();
    for (long j = long(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += long(gridDim.x) * blockDim.x)
        x[j] += a * v[j];
}

__global__ void k_cfg_combine(float* out, const float* vc, const float* vu, float g, long n)
{
    grid_dep_wait();
    grid_dep_launch();
    for (long j = long(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += long(gridDim.x) * blockDim.x)
        out[j] = vu[j] + g * (vc[j] - vu[j]);
}

// x += dt v, then + up * N(0, 1) (engine.cpp:492-499).
__global__ void k_euler_ancestral(float* x, const float* v, float dt, float up, uint64_t key, uint64_t off, long n)
{
    grid_dep_wait();
    grid_dep_launch();
    for (long j = long(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += long(gridDim.x) * blockDim.x) {
        float xv = x[j] + dt * v[j];
        if (up > 0.f)
            xv += up * float(counter_normal(key, off + uint64_t(j)));
        x[j] = xv;
    }
}

struct ErSdeArgs {
    double c1, c2, c3, c4, d_den, u_den, cn;
    float sigma;  // sigma_i: the image estimate is x - sigma_i v (engine.cpp:483-486)
    int stage, last, noise;
};

// One ER-SDE step (er_sde.cpp:27-74) on x; state holds the previous image estimate [n] and difference [n].
__global__ void k_er_sde(float* x, const float* v, float* old, float* old_d, ErSdeArgs a, uint64_t key, uint64_t off,
                         long n)
{
    grid_dep_wait();
    grid_dep_launch();
    for (long j = long(blockIdx.x) * blockDim.x + threadIdx.x; j < n; j += long(gridDim.x) * blockDim.x) {
        const float den = x[j] - a.sigma * v[j];
        if (a.last) {
            x[j] = den;
        } else {
            double val = a.c1 * x[j] + a.c2 * den;
            if (a.stage >= 2) {
                const double d = (double(den) - old[j]) / a.d_den;
                val += a.c3 * d;
                if (a.stage >= 3)
                    val += a.c4 * (d - old_d[j]) / a.u_den;
                old_d[j] = float(d);
            }
            if (a.noise)
                val += a.cn * float(counter_normal(key, off + uint64_t(j)));
            x[j] = float(val);
        }
        old[j] = den;
    }
}

}  // namespace

}  // namespace mkb

using namespace mkb;

extern "C" {

mkb_status mkb_cfg_combine_dev(float* out, const float* v_cond, const float* v_uncond, float guidance, long n,
                               void* stream)
{
    if (!out || !v_cond || !v_uncond || n <= 0)
        return fail(MKB_ERR_INVALID, "cfg_combine: bad arguments");
    launch_k(k_cfg_combine, grid_of(n), 256, 0, static_cast<cudaStream_t>(stream), out, v_cond, v_uncond, guidance,
             n);
    count_launch();
    return cuda_status(cudaGetLastError(), "cfg_combine launch");
}

mkb_status mkb_axpy_dev(float* x, const float* v, float a, long n, void* stream)
{
    if (!x || !v || n <= 0)
        return fail(MKB_ERR_INVALID, "axpy: bad arguments");
    launch_k(k_axpy, grid_of(n), 256, 0, static_cast<cudaStream_t>(stream), x, v, a, n);
    count_launch();
    return cuda_status(cudaGetLastError(), "axpy launch");
}

mkb_status mkb_euler_ancestral_dev(float* x, const float* v, float sigma, float sigma_next, uint64_t noise_key,
                                   uint64_t noise_offset, long n, void* stream)
{
    if (!x || !v || n <= 0 || !(sigma > 0.f) || sigma_next < 0.f || sigma_next > sigma)
        return fail(MKB_ERR_INVALID, "euler_ancestral: bad arguments (need sigma > 0 and 0 <= sigma_next <= sigma)");
    // Down to the level whose noise, with fresh noise of the remainder added, makes the next one's.
    const double from = sigma, to = sigma_next;
    const double up = std::min(to, std::sqrt(to * to * (from * from - to * to) / (from * from)));
    const float dt = float(std::sqrt(to * to - up * up) - from);
    launch_k(k_euler_ancestral, grid_of(n), 256, 0, static_cast<cudaStream_t>(stream), x, v, dt, float(up),
             noise_key, noise_offset, n);
    count_launch();
    return cuda_status(cudaGetLastError(), "euler_ancestral launch");
}

mkb_status mkb_er_sde_step_dev(mkb_er_sde* e, int i, float* x, const float* v, float* state, uint64_t noise_key,
                               uint64_t noise_offset, long n, float s_noise, void* stream)
{
    if (!e || !x || !v || !state || n <= 0)
        return fail(MKB_ERR_INVALID, "er_sde_step_dev: bad arguments");
    ErSdeCoef c;
    if (!er_sde_coef(e, i, s_noise, &c))
        return fail(MKB_ERR_INVALID, "er_sde_step_dev: step out of range");
    if (!er_sde_dev_order(e, i))
        return fail(MKB_ERR_STATE, "er_sde_step_dev: steps of a run must go 0, 1, 2, ...");
    ErSdeArgs a{c.c1, c.c2, c.c3, c.c4, c.d_den, c.u_den, c.cn, float(er_sde_sigma_d(e, i)), c.stage,
                c.last ? 1 : 0, s_noise > 0.f ? 1 : 0};
    launch_k(k_er_sde, grid_of(n), 256, 0, static_cast<cudaStream_t>(stream), x, v, state, state + n, a,
             noise_key, noise_offset, n);
    count_launch();
    return cuda_status(cudaGetLastError(), "er_sde launch");
}

}  // extern "C"
