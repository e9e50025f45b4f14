// C entry points over the reference's own image::ErSde (src/image/er_sde.cpp), compiled from the reference's source
// tree by oracle/Makefile into oracle/_ref/liber_sde_ref.so. TEST INFRASTRUCTURE ONLY: the tests call it to pin the
// oracle's ER-SDE restatement and the library's sampler to the reference's behaviour.
#include "image/er_sde.hpp"

#include <span>
#include <vector>

extern "C" {

void* ref_er_sde_create(const float* sigmas, int n, int flow, float top)
{
    return new mako::image::ErSde(std::span<const float>(sigmas, size_t(n)), flow != 0, top);
}

void ref_er_sde_destroy(void* e) { delete static_cast<mako::image::ErSde*>(e); }

float ref_er_sde_sigma(void* e, int i) { return static_cast<mako::image::ErSde*>(e)->sigma(uint32_t(i)); }

void ref_er_sde_step(void* e, int i, float* x, const float* den, const float* noise, long n, float s_noise)
{
    static_cast<mako::image::ErSde*>(e)->step(uint32_t(i), std::span<float>(x, size_t(n)),
                                              std::span<const float>(den, size_t(n)),
                                              std::span<const float>(noise, size_t(n)), s_noise);
}
}
