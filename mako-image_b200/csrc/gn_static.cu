// GroupNorm without a caller-supplied workspace: the statistics scratch lives in this library's own device memory.
//
// mkb_group_norm needs scratch memory for its per-chunk statistics, and its callers pass it in. Some callers have no
// way to do that: code that runs while another component owns all device memory (a serving loop whose caching
// allocator must not be bypassed), real-time paths where an allocation's latency or possible failure is not
// acceptable, and hosts that only hand this library tensors they already own. mkb_group_norm_static serves them: its
// scratch is a fixed array compiled into the library, so the call allocates nothing.
#include "common.cuh"
#include "rowops.cuh"

#include <mutex>
#include <string>

namespace mkb {

namespace {

// The statistics scratch: kStaticGnBytes on every device that loads the library, kept until the process exits.
constexpr size_t kStaticGnBytes = size_t(4) << 20;
static __device__ __align__(256) unsigned char g_gn_scratch[kStaticGnBytes];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

// The device address of g_gn_scratch on the current device, looked up once per device. In host code the symbol is a
// host-side stand-in, not a device address, so it is never passed to a kernel itself. The cached address assumes the
// device's primary context lives until the process exits: after cudaDeviceReset (or a release and re-creation of the
// primary context) the module can load at another address, and this entry point must not be used again on that
// device.
mkb_status scratch_address(void** out)
{
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess)
        return cuda_status(e, "group_norm_static: current device");
    if (dev < 0 || dev >= kMaxDevices)
        return fail(MKB_ERR_INVALID, "group_norm_static: device index out of range");
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_gn_scratch);
        if (e != cudaSuccess)
            return cuda_status(e, "group_norm_static: scratch address");
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return MKB_OK;
}

}  // namespace

}  // namespace mkb

using namespace mkb;

extern "C" {

size_t mkb_group_norm_static_max_bytes(void) { return kStaticGnBytes; }

mkb_status mkb_group_norm_static(const float* x, void* y, const float* gamma, const float* beta, int B, int HW, int C,
                                 int groups, float eps, int silu, void* stream)
{
    if (!x || !y || !gamma)
        return fail(MKB_ERR_INVALID, "group_norm_static: null argument");
    if (B <= 0 || HW <= 0 || groups <= 0 || C % groups || C % 4 || C > 6144)
        return fail(MKB_ERR_INVALID, "group_norm_static: need C a multiple of groups and of 4, C <= 6144");
    const size_t need = group_norm_workspace(B, HW, C, groups);
    if (need > kStaticGnBytes)
        return fail(MKB_ERR_INVALID, "group_norm_static: these sizes need " + std::to_string(need) +
                                         " bytes of statistics scratch, above the built-in " +
                                         std::to_string(kStaticGnBytes) + "; use mkb_group_norm with a workspace");
    void* ws = nullptr;
    mkb_status s = scratch_address(&ws);
    if (s != MKB_OK)
        return s;
    // Every entry the kernels read is written earlier in the same call (the per-chunk statistics, then the per-group
    // mean and scale), so the previous call's contents need no clearing.
    GnArgs a{x, static_cast<__nv_bfloat16*>(y), gamma, beta, B, HW, C, groups, eps, silu, static_cast<float*>(ws)};
    return cuda_status(group_norm(a, static_cast<cudaStream_t>(stream)), "group_norm_static launch");
}

}  // extern "C"
