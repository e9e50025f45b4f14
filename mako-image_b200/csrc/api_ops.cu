// The runtime-operation layer of the C ABI (include/mkb_image.h, part 1): argument checks, then one prepared
// kernel launch each.
#include "common.cuh"
#include "launch.cuh"
#include "attention.cuh"
#include "gemm.cuh"
#include "rowops.cuh"
#include "sm100.cuh"

#include <algorithm>
#include <atomic>
#include <cstdlib>
#include <mutex>
#include <string>
#include <vector>

namespace mkb {

namespace {
thread_local std::string g_last_error;
std::atomic<unsigned long long> g_launches{0};
std::mutex g_status_mu;
std::vector<uint32_t*> g_status_words;  // per device
}  // namespace

void count_launch(unsigned long long n) { g_launches.fetch_add(n, std::memory_order_relaxed); }

bool pdl_enabled()
{
    static const bool on = [] {
        const char* v = std::getenv("MKB_PDL");
        return !(v && v[0] == '0');
    }();
    return on;
}

mkb_status fail(mkb_status code, const std::string& msg)
{
    g_last_error = msg;
    return code;
}

mkb_status cuda_status(cudaError_t e, const char* what)
{
    if (e == cudaSuccess)
        return MKB_OK;
    // The error is reported here; clear the thread's last-error state so a later launch check does not report a
    // non-sticky one (a failed allocation) a second time.
    cudaGetLastError();
    return fail(e == cudaErrorMemoryAllocation ? MKB_ERR_ALLOC : MKB_ERR_CUDA,
                std::string(what) + ": " + cudaGetErrorString(e));
}

uint32_t* device_status_word()
{
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess)
        return nullptr;
    std::lock_guard<std::mutex> lk(g_status_mu);
    if (int(g_status_words.size()) <= dev)
        g_status_words.resize(dev + 1, nullptr);
    if (!g_status_words[dev]) {
        uint32_t* p = nullptr;
        if (cudaMalloc(&p, sizeof(uint32_t)) != cudaSuccess) {
            cudaGetLastError();
            return nullptr;
        }
        cudaMemset(p, 0, sizeof(uint32_t));
        g_status_words[dev] = p;
    }
    return g_status_words[dev];
}

namespace {

mkb_status run_gemm(Epi epi, const void* x, long ldx, const void* w, long ldw, GemmArgs a, int bn, void* stream)
{
    if (!x || !w)
        return fail(MKB_ERR_INVALID, "proj: null operand");
    a.status = device_status_word();
    GemmOp op;
    const char* err = nullptr;
    if (!gemm_prepare(op, epi, x, ldx, w, ldw, a, bn, &err))
        return fail(MKB_ERR_INVALID, err ? err : "proj: unsupported arguments");
    // CTA pairs when the makespan estimate prefers them at this width: the pair halves each SM's W traffic.
    if (bn >= 128 && gemm_pick_tile(a.M, a.N, true, bn).pairs && !gemm_use_pairs(op, &err))
        return fail(MKB_ERR_INVALID, err ? err : "proj: pair set-up failed");
    return cuda_status(gemm_launch(op, static_cast<cudaStream_t>(stream)), "proj launch");
}

int pick_bn(int M, int N) { return gemm_pick_tile(M, N, true).bn; }

}  // namespace

}  // namespace mkb

using namespace mkb;

extern "C" {

const char* mkb_last_error(void) { return g_last_error.c_str(); }

uint64_t mkb_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

mkb_status mkb_proj(const void* x, long ldx, const void* w, long ldw, const float* bias, void* y, long ldy, int M,
                    int N, int K, int act, int out_f32, void* stream)
{
    if (act < MKB_ACT_NONE || act > MKB_ACT_GELU_ERF)
        return fail(MKB_ERR_INVALID, "proj: unknown activation");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.act = act;
    a.out = y;
    a.ldo = ldy;
    return run_gemm(out_f32 ? Epi::kF32 : Epi::kBF16, x, ldx, w, ldw, a, pick_bn(M, N), stream);
}

mkb_status mkb_proj_gate_add(const void* x, long ldx, const void* w, long ldw, const float* bias, float* resid,
                             long ldr, const float* gate, long gate_stride, int rows_per_sample, int tanh_gate, int M,
                             int N, int K, void* stream)
{
    if (rows_per_sample <= 0)
        return fail(MKB_ERR_INVALID, "proj_gate_add: rows_per_sample must be positive");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.resid = resid;
    a.ldr = ldr;
    a.gate = gate;
    a.gate_bstride = gate_stride;
    a.seg_rows = rows_per_sample;
    a.tanh_gate = tanh_gate;
    return run_gemm(Epi::kResid, x, ldx, w, ldw, a, pick_bn(M, N), stream);
}

mkb_status mkb_proj_qkv_heads(const void* x, long ldx, const void* w, long ldw, const float* bias,
                              const float* norm_q, const float* norm_k, const float* rope, void* qh, void* kh,
                              void* vh, int heads, int L, int rows_per_sample, int pos_offset, float eps, int M, int K,
                              void* stream)
{
    if (heads <= 0 || L <= 0 || rows_per_sample <= 0 || pos_offset < 0 || pos_offset + rows_per_sample > L)
        return fail(MKB_ERR_INVALID, "proj_qkv_heads: need heads > 0 and pos_offset + rows_per_sample <= L");
    if (!norm_q || !norm_k)
        return fail(MKB_ERR_INVALID, "proj_qkv_heads: null norm weights");
    GemmArgs a;
    a.M = M;
    a.D = heads * 128;
    a.N = 3 * a.D;
    a.K = K;
    a.bias = bias;
    a.qh = static_cast<__nv_bfloat16*>(qh);
    a.kh = static_cast<__nv_bfloat16*>(kh);
    a.vh = static_cast<__nv_bfloat16*>(vh);
    a.norm_q = norm_q;
    a.norm_k = norm_k;
    a.rope = rope;
    a.L = L;
    a.seg_rows = rows_per_sample;
    a.seg_off = pos_offset;
    a.eps = eps;
    const int bn = (a.D % 256 == 0) ? 256 : 128;
    return run_gemm(Epi::kQkv, x, ldx, w, ldw, a, bn, stream);
}

int mkb_swiglu_interleave(void) { return 128; }

mkb_status mkb_proj_swiglu(const void* x, long ldx, const void* w, long ldw, const float* bias, void* y, long ldy,
                           int M, int N, int K, void* stream)
{
    if (N % 256)
        return fail(MKB_ERR_INVALID, "proj_swiglu: N (gate + up rows) must be a multiple of 256");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.out = y;
    a.ldo = ldy;
    return run_gemm(Epi::kSwiGLU, x, ldx, w, ldw, a, 256, stream);
}

mkb_status mkb_proj_add(const void* x, long ldx, const void* w, long ldw, const float* bias, const float* addvec,
                        long addvec_stride, int rows_per_sample, const float* resid, long ld_resid, void* y, long ldy,
                        int out_f32, int M, int N, int K, void* stream)
{
    if (addvec && rows_per_sample <= 0)
        return fail(MKB_ERR_INVALID, "proj_add: rows_per_sample must be positive");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.addvec = addvec;
    a.addvec_stride = addvec_stride;
    a.seg_rows = addvec ? rows_per_sample : (1 << 30);
    a.add_resid = resid;
    a.ld_add_resid = ld_resid;
    a.out = y;
    a.ldo = ldy;
    a.out_f32 = out_f32;
    return run_gemm(Epi::kAdd, x, ldx, w, ldw, a, pick_bn(M, N), stream);
}

mkb_status mkb_proj_heads(const void* x, long ldx, const void* w, long ldw, const float* bias, void* qh, void* kh,
                          void* vh, int part0, int D, int head_dim, int L, int rows_per_sample, int pos_offset, int M,
                          int N, int K, void* stream)
{
    if (rows_per_sample <= 0 || pos_offset < 0 || pos_offset + rows_per_sample > L || D <= 0)
        return fail(MKB_ERR_INVALID, "proj_heads: need pos_offset + rows_per_sample <= L and D > 0");
    const int parts = (N + D - 1) / D;
    void* outs[3] = {qh, kh, vh};
    for (int p = part0; p < part0 + parts && p < 3; ++p)
        if (!outs[p])
            return fail(MKB_ERR_INVALID, "proj_heads: missing output for a part");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.qh = static_cast<__nv_bfloat16*>(qh);
    a.kh = static_cast<__nv_bfloat16*>(kh);
    a.vh = static_cast<__nv_bfloat16*>(vh);
    a.part0 = part0;
    a.D = D;
    a.head_dim = head_dim;
    a.L = L;
    a.seg_rows = rows_per_sample;
    a.seg_off = pos_offset;
    return run_gemm(Epi::kHeads, x, ldx, w, ldw, a, pick_bn(M, N), stream);
}

mkb_status mkb_proj_geglu(const void* x, long ldx, const void* w, long ldw, const float* bias, void* y, long ldy,
                          int M, int N, int K, void* stream)
{
    if (N % 256)
        return fail(MKB_ERR_INVALID, "proj_geglu: N (hidden + gate rows) must be a multiple of 256");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.bias = bias;
    a.out = y;
    a.ldo = ldy;
    a.glu = kGluGelu;
    return run_gemm(Epi::kSwiGLU, x, ldx, w, ldw, a, 256, stream);
}

mkb_status mkb_conv2d(const void* x, int B, int H, int W, int C, const void* w, int Cout, int taps, int stride,
                      const float* bias, const float* addvec, long addvec_stride, const float* resid, long ld_resid,
                      void* y, long ldy, int out_f32, void* stream)
{
    if (!x || !w || !y)
        return fail(MKB_ERR_INVALID, "conv2d: null operand");
    GemmArgs a;
    a.bias = bias;
    a.addvec = addvec;
    a.addvec_stride = addvec_stride;
    a.add_resid = resid;
    a.ld_add_resid = ld_resid;
    a.out = y;
    a.ldo = ldy;
    a.out_f32 = out_f32;
    a.status = device_status_word();
    const int Ho = taps == 9 ? (H - 1) / stride + 1 : H, Wo = taps == 9 ? (W - 1) / stride + 1 : W;
    const GemmTile t = gemm_pick_tile(long(B) * Ho * Wo, Cout, true);
    GemmOp op;
    const char* err = nullptr;
    if (!conv_prepare(op, Epi::kAdd, x, B, H, W, C, w, Cout, taps, stride, a, t.bn, &err))
        return fail(MKB_ERR_INVALID, err ? err : "conv2d: unsupported arguments");
    if (t.pairs && !gemm_use_pairs(op, &err))
        return fail(MKB_ERR_INVALID, err ? err : "conv2d: pair set-up failed");
    return cuda_status(gemm_launch(op, static_cast<cudaStream_t>(stream)), "conv2d launch");
}

mkb_status mkb_ln_modulate(const float* x, const float* mod, const float* shift, void* y, long rows, int n, float eps,
                           long split, long mod_stride, long mod_off, void* stream)
{
    if (!x || !mod || !y || rows < 0 || rows > (1L << 30) || n <= 0 || n % 128 || n > 4096)
        return fail(MKB_ERR_INVALID, "ln_modulate: need rows >= 0 and n a multiple of 128 up to 4096");
    if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(mod + mod_off) & 15) ||
        (shift && (reinterpret_cast<uintptr_t>(shift + mod_off) & 15)) || (mod_stride & 3) ||
        (reinterpret_cast<uintptr_t>(y) & 7))
        return fail(MKB_ERR_INVALID, "ln_modulate: x, mod + mod_off, shift + mod_off need 16-byte alignment");
    LnModArgs a{};
    a.x = x;
    a.y = static_cast<__nv_bfloat16*>(y);
    a.scale = mod + mod_off;
    a.shift = shift ? shift + mod_off : nullptr;
    a.mod_stride = 0;
    a.alt_off = mod_stride;  // rows before split read the second modulation row
    a.split = int(std::min(std::max(split, 0L), rows));
    a.rows = int(rows);
    a.D = n;
    a.rows_per_sample = rows > 0 ? int(rows) : 1;
    a.eps = eps;
    return cuda_status(ln_modulate(a, static_cast<cudaStream_t>(stream)), "ln_modulate");
}

size_t mkb_group_norm_workspace_size(int B, int HW, int C, int groups)
{
    return group_norm_workspace(B, HW, C, groups);
}

mkb_status mkb_group_norm(const float* x, void* y, const float* gamma, const float* beta, int B, int HW, int C,
                          int groups, float eps, int silu, void* workspace, size_t workspace_bytes, void* stream)
{
    if (!x || !y || !gamma || !workspace)
        return fail(MKB_ERR_INVALID, "group_norm: null argument");
    if (B <= 0 || HW <= 0 || groups <= 0 || C % groups || C % 4 || C > 6144)
        return fail(MKB_ERR_INVALID, "group_norm: need C a multiple of groups and of 4, C <= 6144");
    if (workspace_bytes < group_norm_workspace(B, HW, C, groups))
        return fail(MKB_ERR_INVALID, "group_norm: workspace too small");
    GnArgs a{x, static_cast<__nv_bfloat16*>(y), gamma, beta, B, HW, C, groups, eps, silu,
             static_cast<float*>(workspace)};
    return cuda_status(group_norm(a, static_cast<cudaStream_t>(stream)), "group_norm launch");
}

mkb_status mkb_attention(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk, int Lk_rows, int B,
                         int H, int head_dim, int q_pos0, int mask, int cond_len, int split, void* out0, long ld0,
                         int rows0, void* out1, long ld1, int rows1, void* stream)
{
    return mkb_attention_kv_shards(q, Lq, Lq_rows, k, v, Lk, Lk_rows, B, H, head_dim, q_pos0, mask, cond_len, split,
                                   out0, ld0, rows0, out1, ld1, rows1, 0, 0, stream);
}

mkb_status mkb_attention_wide(const void* qkv, long ld, int n, int d, int q_col, int k_col, int v_col, void* out,
                              long ldo, void* stream)
{
    if (!qkv || !out)
        return fail(MKB_ERR_INVALID, "attention_wide: null buffer");
    AttnWideArgs a;
    a.n = n;
    a.d = d;
    a.q_col = q_col;
    a.k_col = k_col;
    a.v_col = v_col;
    a.out = static_cast<__nv_bfloat16*>(out);
    a.ldo = ldo;
    a.scale_log2 = 1.4426950408889634f / sqrtf(float(d));
    a.status = device_status_word();
    AttnWideOp op;
    const char* err = nullptr;
    if (!attn_wide_prepare(op, qkv, ld, a, &err))
        return fail(MKB_ERR_INVALID, err ? err : "attention_wide: unsupported arguments");
    return cuda_status(attn_wide_launch(op, static_cast<cudaStream_t>(stream)), "attention_wide launch");
}

mkb_status mkb_attention_kv_shards(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk,
                                   int Lk_rows, int B, int H, int head_dim, int q_pos0, int mask, int cond_len,
                                   int split, void* out0, long ld0, int rows0, void* out1, long ld1, int rows1,
                                   int kv_shard_rows, int kv_plane_stride, void* stream)
{
    return mkb_attention_kv_arriving(q, Lq, Lq_rows, k, v, Lk, Lk_rows, B, H, head_dim, q_pos0, mask, cond_len, split,
                                     out0, ld0, rows0, out1, ld1, rows1, kv_shard_rows, kv_plane_stride, -1, nullptr,
                                     nullptr, stream);
}

mkb_status mkb_attention_kv_arriving(const void* q, int Lq, int Lq_rows, const void* k, const void* v, int Lk,
                                     int Lk_rows, int B, int H, int head_dim, int q_pos0, int mask, int cond_len,
                                     int split, void* out0, long ld0, int rows0, void* out1, long ld1, int rows1,
                                     int kv_shard_rows, int kv_plane_stride, int own_shard,
                                     const unsigned long long* shard_ready, const unsigned long long* shard_expect,
                                     void* stream)
{
    if (!q || !k || !v)
        return fail(MKB_ERR_INVALID, "attention: null q/k/v");
    if (mask != MKB_MASK_NONE && mask != MKB_MASK_COND_CAUSAL)
        return fail(MKB_ERR_INVALID, "attention: unknown mask");
    AttnArgs a;
    a.B = B;
    a.H = H;
    a.Lq = Lq;
    a.Lk = Lk;
    a.q_pos0 = q_pos0;
    a.mask = mask;
    a.cond_len = cond_len;
    a.head_dim = head_dim;
    a.scale_log2 = 1.4426950408889634f / sqrtf(float(head_dim));
    a.split = split;
    a.out0 = static_cast<__nv_bfloat16*>(out0);
    a.ld0 = ld0;
    a.rows0 = rows0;
    a.out1 = static_cast<__nv_bfloat16*>(out1);
    a.ld1 = ld1;
    a.rows1 = rows1;
    a.kv_shard_rows = kv_shard_rows;
    a.kv_plane_stride = kv_plane_stride;
    a.own_shard = own_shard < 0 ? -1 : own_shard;
    a.shard_ready = shard_ready;
    a.shard_expect = shard_expect;
    a.status = device_status_word();
    AttnOp op;
    const char* err = nullptr;
    if (!attn_prepare(op, q, Lq_rows, k, v, Lk_rows, a, &err))
        return fail(MKB_ERR_INVALID, err ? err : "attention: unsupported arguments");
    return cuda_status(attn_launch(op, static_cast<cudaStream_t>(stream)), "attention launch");
}

mkb_status mkb_selftest_stalled_gemm(const void* x, long ldx, const void* w, long ldw, float* y, long ldy, int M,
                                     int N, int K, void* stream)
{
    if (!x || !w || !y)
        return fail(MKB_ERR_INVALID, "selftest: null operand");
    GemmArgs a;
    a.M = M;
    a.N = N;
    a.K = K;
    a.out = y;
    a.ldo = ldy;
    a.status = device_status_word();
    GemmOp op;
    const char* err = nullptr;
    if (!gemm_prepare(op, Epi::kF32, x, ldx, w, ldw, a, 128, &err))
        return fail(MKB_ERR_INVALID, err ? err : "selftest: unsupported arguments");
    op.p.test_stall = 1;  // the 1-CTA kernel: CTA 0 withholds its first stage's load
    return cuda_status(gemm_launch(op, static_cast<cudaStream_t>(stream)), "selftest launch");
}

mkb_status mkb_check_kernels(uint32_t* bits)
{
    uint32_t* st = device_status_word();
    if (!st)
        return fail(MKB_ERR_CUDA, "status word unavailable");
    MKB_TRY_CUDA(cudaDeviceSynchronize(), "synchronize");
    uint32_t v = 0;
    MKB_TRY_CUDA(cudaMemcpy(&v, st, sizeof(v), cudaMemcpyDeviceToHost), "read status");
    if (bits)
        *bits = v;
    if (v) {
        cudaMemset(st, 0, sizeof(uint32_t));
        return fail(MKB_ERR_KERNEL, "kernel status bits 0x" + std::to_string(v));
    }
    return MKB_OK;
}

}  // extern "C"
