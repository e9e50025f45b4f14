// The counter-based normal generator shared by the synthetic-input fill and the device samplers: element e of the
// stream `key` comes from splitmix64(key + e / 2) by the Box-Muller transform (even e: cos, odd e: sin branch), so
// any slice is produced independently and the numpy oracle reproduces it.
#pragma once

#include <cstdint>

namespace mkb {

__device__ __forceinline__ uint64_t splitmix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ double counter_normal(uint64_t key, uint64_t e)
{
    const uint64_t h = splitmix64(key + (e >> 1));
    const double u1 = (double(h >> 40) + 0.5) / 16777216.0;
    const double u2 = double(h & 0xFFFFFFull) / 16777216.0;
    const double rr = sqrt(-2.0 * log(u1));
    const double ang = 6.283185307179586 * u2;
    return (e & 1) ? rr * sin(ang) : rr * cos(ang);
}

}  // namespace mkb
