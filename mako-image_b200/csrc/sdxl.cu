// The SDXL UNet step and the SDXL (AutoencoderKL) VAE decoder behind include/mkb_image.h part 3.
//
// The UNet follows Sdxl::begin / step (src/image/sdxl.cpp:672-953), the VAE Engine::decode (engine.cpp:862-954).
// Every convolution is the tcgen05 implicit GEMM (csrc/gemm.cu conv mode) with bias, the per-image time embedding
// and the residual fused into its epilogue; GroupNorm(+SiLU) is one two-pass kernel producing the next conv's bf16
// input; transformer blocks use the projection epilogues (head scatter, GEGLU, in-place residual add) and the hd-64
// flash attention; the VAE's single-head d=512 mid attention is two GEMMs around a row softmax, in query chunks.
// A plan (the launch sequence of one geometry) is built once, then captured and replayed as a CUDA graph.
#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "lora.cuh"
#include "rowops.cuh"

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

namespace mkb {

namespace {

// Whether the VAE's convolutions leave the GroupNorm statistics of their outputs (MKB_GN_FUSED=0: the three-pass
// GroupNorm everywhere, for comparison; the statistics need the TMA epilogue, so MKB_TMA_EPI=0 turns them off too).
bool vae_flash_enabled()  // MKB_VAE_FLASH=0: the mid attention as score GEMMs, row softmax and P V GEMMs
{
    static const bool on = [] {
        const char* f = std::getenv("MKB_VAE_FLASH");
        return !(f && f[0] == '0');
    }();
    return on;
}

bool gn_fused_enabled()
{
    static const bool on = [] {
        const char* f = std::getenv("MKB_GN_FUSED");
        const char* t = std::getenv("MKB_TMA_EPI");
        return !(f && f[0] == '0') && !(t && t[0] == '0');
    }();
    return on;
}


constexpr int kHead = 64, kTime = 256, kAdded6 = 6 * 256;
constexpr int kGluBlock = 128;

uint64_t mix64(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

// ------------------------------------------------------------------------------------------------ weight table

// Weights with a logical host layout and a device layout that may pad or interleave:
//   vec    fp32 [r]                              (device: r rounded up to rp, zeros beyond r)
//   mat    bf16 [r][c] -> [rp][cp]               (zero rows / columns beyond r / c)
//   conv3  bf16 [r][3][3][c] -> [rp][9][cp]      (3x3 convolution, tap-major, input channels padded)
//   glu    bf16 [r][c], r = 2F (first half / second half) -> rows interleaved in blocks of 128 for the GLU epilogue
//   gluvec fp32 [r], the bias of a glu matrix, interleaved the same way (the GLU epilogue reads bias by device column)
//   matdup bf16 [r][c] -> [r][2c], the matrix twice along K: against an input split into a bf16 part and the bf16
//          rounding of its remainder ([hi | lo], K = 2c), one GEMM multiplies the fp32 input
//   tab    fp32 [r][c] (embedding tables and other fp32 matrices)
struct WTable {
    enum Kind { kVec, kMat, kConv3, kGlu, kGluVec, kMatDup, kTab };
    static bool is_vec(Kind k) { return k == kVec || k == kGluVec || k == kTab; }
    struct W {
        std::string name;
        Kind kind;
        long r, c, rp, cp;
        size_t off;
        bool norm;
        size_t dev_count() const
        {
            if (kind == kTab)
                return size_t(r) * c;
            if (kind == kMatDup)
                return size_t(rp) * 2 * cp;
            return is_vec(kind) ? size_t(rp) : kind == kConv3 ? size_t(rp) * 9 * cp : size_t(rp) * cp;
        }
        long dev_cols() const { return kind == kMatDup ? 2 * cp : cp; }  // row stride of a matrix on the device
    };
    std::vector<W> ws;
    std::map<std::string, int> idx;
    size_t nmat = 0, nvec = 0;
    __nv_bfloat16* mat = nullptr;
    float* vec = nullptr;

    void add(const std::string& name, Kind k, long r, long c = 0, long rp = 0, long cp = 0, bool norm = false)
    {
        W w{name, k, r, c, rp ? rp : r, cp ? cp : c, 0, norm};
        if (is_vec(k)) {
            if (k != kTab)
                w.rp = (w.rp + 3) & ~3L;
            w.off = nvec;
            nvec += (w.dev_count() + 3) & ~size_t(3);
        } else {
            w.off = nmat;
            nmat += (w.dev_count() + 7) & ~size_t(7);  // 16-byte aligned starts
        }
        idx[name] = int(ws.size());
        ws.push_back(w);
    }
    const W* find(const std::string& n) const
    {
        auto it = idx.find(n);
        return it == idx.end() ? nullptr : &ws[it->second];
    }
    const __nv_bfloat16* M(const std::string& n) const
    {
        const W* w = find(n);
        return w ? mat + w->off : nullptr;
    }
    const float* V(const std::string& n) const
    {
        const W* w = find(n);
        return w ? vec + w->off : nullptr;
    }
    mkb_status alloc()
    {
        MKB_TRY_CUDA(cudaMalloc(&mat, nmat * 2 + 16), "weights");
        MKB_TRY_CUDA(cudaMalloc(&vec, nvec * 4 + 16), "weights");
        MKB_TRY_CUDA(cudaMemset(mat, 0, nmat * 2 + 16), "weights");
        MKB_TRY_CUDA(cudaMemset(vec, 0, nvec * 4 + 16), "weights");
        return MKB_OK;
    }
    void release()
    {
        if (mat)
            cudaFree(mat);
        if (vec)
            cudaFree(vec);
        mat = nullptr;
        vec = nullptr;
    }
    // Device row of logical row i of a glu matrix with 2F rows.
    static long glu_row(long i, long rows)
    {
        const long F = rows / 2;
        const bool second = i >= F;
        const long j = second ? i - F : i;
        return (j / kGluBlock) * 2 * kGluBlock + (second ? kGluBlock : 0) + j % kGluBlock;
    }
    mkb_status init_random(uint64_t seed, float std, cudaStream_t s)
    {
        for (size_t i = 0; i < ws.size(); ++i) {
            const W& w = ws[i];
            const uint64_t key = mix64(seed * 0x100000001B3ull + i);
            const float sd = w.norm ? 0.1f : std, mean = w.norm ? 1.0f : 0.0f;
            if (is_vec(w.kind)) {
                MKB_TRY_CUDA(fill_normal(vec + w.off, false, w.kind == kTab ? w.dev_count() : size_t(w.r), key, 0, sd,
                                         mean, s),
                             "init");
                continue;
            }
            __nv_bfloat16* p = mat + w.off;
            MKB_TRY_CUDA(fill_normal(p, true, w.dev_count(), key, 0, sd, mean, s), "init");
            if (w.kind == kMatDup) {  // the second copy along K equals the first
                MKB_TRY_CUDA(cudaMemcpy2DAsync(p + w.cp, size_t(w.cp) * 4, p, size_t(w.cp) * 4, size_t(w.cp) * 2,
                                               size_t(w.rp), cudaMemcpyDeviceToDevice, s),
                             "init copy");
                continue;
            }
            // padding stays zero
            const long taps = w.kind == kConv3 ? 9 : 1;
            if (w.cp > w.c)
                MKB_TRY_CUDA(cudaMemset2DAsync(p + w.c, size_t(w.cp) * 2, 0, size_t(w.cp - w.c) * 2,
                                               size_t(w.rp) * taps, s),
                             "init pad");
            if (w.rp > w.r)
                MKB_TRY_CUDA(cudaMemsetAsync(p + size_t(w.r) * taps * w.cp, 0, size_t(w.rp - w.r) * taps * w.cp * 2,
                                             s),
                             "init pad");
        }
        MKB_TRY_CUDA(cudaStreamSynchronize(s), "init");
        return MKB_OK;
    }
    mkb_status read(const std::string& name, float* host) const
    {
        const W* w = find(name);
        if (!w || !host)
            return fail(MKB_ERR_INVALID, "weight_read: unknown weight " + name);
        if (w->kind == kVec || w->kind == kTab) {
            MKB_TRY_CUDA(cudaMemcpy(host, vec + w->off, (w->kind == kTab ? w->dev_count() : size_t(w->r)) * 4,
                                    cudaMemcpyDeviceToHost),
                         "weight read");
            return MKB_OK;
        }
        if (w->kind == kGluVec) {
            std::vector<float> t(w->r);
            MKB_TRY_CUDA(cudaMemcpy(t.data(), vec + w->off, w->r * 4, cudaMemcpyDeviceToHost), "weight read");
            for (long i = 0; i < w->r; ++i)
                host[i] = t[glu_row(i, w->r)];
            return MKB_OK;
        }
        std::vector<__nv_bfloat16> t(w->dev_count());
        MKB_TRY_CUDA(cudaMemcpy(t.data(), mat + w->off, t.size() * 2, cudaMemcpyDeviceToHost), "weight read");
        const long taps = w->kind == kConv3 ? 9 : 1, ld = w->dev_cols();
        for (long i = 0; i < w->r; ++i) {
            const long di = w->kind == kGlu ? glu_row(i, w->r) : i;
            for (long k = 0; k < taps; ++k)
                for (long j = 0; j < w->c; ++j)
                    host[(i * taps + k) * w->c + j] = __bfloat162float(t[(size_t(di) * taps + k) * ld + j]);
        }
        return MKB_OK;
    }
    mkb_status write(const std::string& name, const float* host)
    {
        const W* w = find(name);
        if (!w || !host)
            return fail(MKB_ERR_INVALID, "weight_write: unknown weight " + name);
        if (w->kind == kVec || w->kind == kTab) {
            MKB_TRY_CUDA(cudaMemcpy(vec + w->off, host, (w->kind == kTab ? w->dev_count() : size_t(w->r)) * 4,
                                    cudaMemcpyHostToDevice),
                         "weight write");
            return MKB_OK;
        }
        if (w->kind == kGluVec) {
            std::vector<float> t(w->r);
            for (long i = 0; i < w->r; ++i)
                t[glu_row(i, w->r)] = host[i];
            MKB_TRY_CUDA(cudaMemcpy(vec + w->off, t.data(), w->r * 4, cudaMemcpyHostToDevice), "weight write");
            return MKB_OK;
        }
        std::vector<__nv_bfloat16> t(w->dev_count(), __float2bfloat16_rn(0.f));
        const long taps = w->kind == kConv3 ? 9 : 1, ld = w->dev_cols();
        for (long i = 0; i < w->r; ++i) {
            const long di = w->kind == kGlu ? glu_row(i, w->r) : i;
            for (long k = 0; k < taps; ++k)
                for (long j = 0; j < w->c; ++j) {
                    const __nv_bfloat16 v = __float2bfloat16_rn(host[(i * taps + k) * w->c + j]);
                    t[(size_t(di) * taps + k) * ld + j] = v;
                    if (w->kind == kMatDup)
                        t[size_t(di) * ld + w->cp + j] = v;
                }
        }
        MKB_TRY_CUDA(cudaMemcpy(mat + w->off, t.data(), t.size() * 2, cudaMemcpyHostToDevice), "weight write");
        return MKB_OK;
    }
    mkb_status info(int i, const char** name, long* dims, int* ndim) const
    {
        if (i < 0 || i >= int(ws.size()))
            return fail(MKB_ERR_INVALID, "weight_info: index out of range");
        const W& w = ws[i];
        if (name)
            *name = w.name.c_str();
        int n = 0;
        long d[4] = {w.r, 0, 0, 0};
        if (w.kind == kTab) {
            d[1] = w.c;
            n = 2;
        } else if (is_vec(w.kind))
            n = 1;
        else if (w.kind == kConv3) {
            d[1] = 3, d[2] = 3, d[3] = w.c;
            n = 4;
        } else {
            d[1] = w.c;
            n = 2;
        }
        if (dims)
            for (int k = 0; k < 4; ++k)
                dims[k] = d[k];
        if (ndim)
            *ndim = n;
        return MKB_OK;
    }
};

// ------------------------------------------------------------------------------------------------ plans

// The launch sequence of one geometry, with the buffers it owns.
struct Plan {
    std::vector<std::function<cudaError_t(cudaStream_t)>> steps;
    struct Probe {
        size_t after;  // probe after steps[after - 1]
        std::string name;
        int layer;
        const float* p;
        long n;
    };
    std::vector<Probe> probes;
    std::vector<void*> bufs;
    cudaGraphExec_t graph = nullptr;
    int runs = 0;
    unsigned long long launches = 0;
    float* gn_ws = nullptr;
    ~Plan()
    {
        if (graph)
            cudaGraphExecDestroy(graph);
        for (void* b : bufs)
            cudaFree(b);
    }
    template <typename T>
    T* buf(size_t count, mkb_status* st)
    {
        void* p = nullptr;
        if (cudaMalloc(&p, count * sizeof(T) + 256) != cudaSuccess) {
            cudaGetLastError();  // not sticky: keep it out of later launch checks
            *st = fail(MKB_ERR_ALLOC, "sdxl plan: device allocation failed");
            return nullptr;
        }
        bufs.push_back(p);
        return static_cast<T*>(p);
    }
    void add(std::function<cudaError_t(cudaStream_t)> f) { steps.push_back(std::move(f)); }
    void probe(const std::string& name, int layer, const float* p, long n)
    {
        probes.push_back({steps.size(), name, layer, p, n});
    }

    // Runs the sequence eagerly (probing when fn is set), or captured as a CUDA graph from the second run on.
    mkb_status run(cudaStream_t s, mkb_probe_fn fn, void* user)
    {
        if (fn) {
            size_t pi = 0;
            for (size_t i = 0; i <= steps.size(); ++i) {
                for (; pi < probes.size() && probes[pi].after == i; ++pi) {
                    std::vector<float> h(probes[pi].n);
                    MKB_TRY_CUDA(cudaStreamSynchronize(s), "probe");
                    MKB_TRY_CUDA(cudaMemcpy(h.data(), probes[pi].p, h.size() * 4, cudaMemcpyDeviceToHost), "probe");
                    fn(probes[pi].name.c_str(), probes[pi].layer, h.data(), long(h.size()), user);
                }
                if (i < steps.size())
                    MKB_TRY_CUDA(steps[i](s), "sdxl launch");
            }
            return MKB_OK;
        }
        if (graph) {
            MKB_TRY_CUDA(cudaGraphLaunch(graph, s), "graph launch");
            count_launch(launches);
            return MKB_OK;
        }
        if (runs++ == 0) {
            for (auto& f : steps)
                MKB_TRY_CUDA(f(s), "sdxl launch");
            return MKB_OK;
        }
        cudaGraph_t g = nullptr;
        MKB_TRY_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
        const unsigned long long l0 = mkb_kernel_launches();
        cudaError_t err = cudaSuccess;
        for (auto& f : steps)
            if ((err = f(s)) != cudaSuccess)
                break;
        cudaError_t ce = cudaStreamEndCapture(s, &g);
        if (err != cudaSuccess || ce != cudaSuccess) {
            if (g)
                cudaGraphDestroy(g);
            return cuda_status(err != cudaSuccess ? err : ce, "sdxl capture");
        }
        launches = mkb_kernel_launches() - l0;
        ce = cudaGraphInstantiate(&graph, g, 0);
        cudaGraphDestroy(g);
        MKB_TRY_CUDA(ce, "graph instantiate");
        MKB_TRY_CUDA(cudaGraphLaunch(graph, s), "graph launch");
        return MKB_OK;
    }
};

// Helpers that append one fused launch to a plan.
struct Builder {
    Plan& P;
    uint32_t* status;
    const char* err = nullptr;
    mkb_status st = MKB_OK;

    bool ok() const { return st == MKB_OK; }
    void bad(const char* e)
    {
        if (st == MKB_OK)
            st = fail(MKB_ERR_INVALID, std::string("sdxl plan: ") + (e ? e : "unsupported shape"));
    }
    // 3x3 (taps 9) or 1x1 convolution of bf16 x [B][H][W][Cin] into y (fp32 or bf16, row stride ldy) with bias,
    // per-image addvec and fp32 residual.
    // With gn_part the convolution also leaves its output's GroupNorm statistics (32 groups) there, for gn_from().
    void conv(const __nv_bfloat16* x, int B, int H, int W, int Cin, const __nv_bfloat16* w, int Cout, int taps,
              int stride, const float* bias, const float* addvec, long addvec_stride, const float* resid, void* y,
              long ldy, bool out_f32, float4* gn_part = nullptr)
    {
        if (!ok())
            return;
        GemmArgs a;
        if (gn_part) {
            a.gn_part = gn_part;
            a.gn_cpg = Cout / 32;
        }
        a.bias = bias;
        a.addvec = addvec;
        a.addvec_stride = addvec_stride;
        a.add_resid = resid;
        a.ld_add_resid = ldy;
        a.out = y;
        a.ldo = ldy;
        a.out_f32 = out_f32;
        a.status = status;
        const int Ho = stride == 2 ? H / 2 : H, Wo = stride == 2 ? W / 2 : W;
        const GemmTile t = gemm_pick_tile(long(B) * Ho * Wo, Cout, true);
        GemmOp op;
        if (!conv_prepare(op, Epi::kAdd, x, B, H, W, Cin, w, Cout, taps, stride, a, t.bn, &err))
            return bad(err);
        if (t.pairs && !gemm_use_pairs(op, &err))
            return bad(err);
        P.add([op](cudaStream_t s) { return gemm_launch(op, s); });
    }
    void gemm(Epi epi, const void* x, long ldx, const void* w, long ldw, GemmArgs a, int bn = 0)
    {
        if (!ok())
            return;
        a.status = status;
        GemmTile t{bn, false};
        if (epi == Epi::kSwiGLU)
            t = gemm_pick_tile(a.M, a.N, true, 256);
        else if (!bn)
            t = gemm_pick_tile(a.M, a.N, true);
        GemmOp op;
        if (!gemm_prepare(op, epi, x, ldx, w, ldw, a, t.bn, &err))
            return bad(err);
        if (t.pairs && !gemm_use_pairs(op, &err))
            return bad(err);
        P.add([op](cudaStream_t s) { return gemm_launch(op, s); });
    }
    void gn(const float* x, __nv_bfloat16* y, const float* g, const float* b, int B, int HW, int C, float eps,
            bool silu)
    {
        if (!ok())
            return;
        GnArgs a{x, y, g, b, B, HW, C, 32, eps, silu ? 1 : 0, P.gn_ws};
        P.add([a](cudaStream_t s) { return group_norm(a, s); });
    }
    // GroupNorm of x whose statistics the convolution that wrote it left in parts (nchunks per image and group).
    void gn_from(const float* x, const float4* parts, int nchunks, __nv_bfloat16* y, const float* g, const float* b,
                 int B, int HW, int C, float eps, bool silu)
    {
        if (!ok())
            return;
        GnArgs a{x, y, g, b, B, HW, C, 32, eps, silu ? 1 : 0, P.gn_ws};
        P.add([a, parts, nchunks](cudaStream_t s) { return group_norm_from_parts(a, parts, nchunks, s); });
    }
    void attn(const __nv_bfloat16* q, const __nv_bfloat16* k, const __nv_bfloat16* v, int B, int H, int Lq, int Lk,
              __nv_bfloat16* out, int hd = kHead)
    {
        if (!ok())
            return;
        AttnArgs a;
        a.B = B;
        a.H = H;
        a.Lq = Lq;
        a.Lk = Lk;
        a.head_dim = hd;
        a.scale_log2 = 1.4426950408889634f / std::sqrt(float(hd));
        a.split = 0;
        a.out1 = out;
        a.ld1 = long(H) * hd;
        a.rows1 = Lq;
        a.status = status;
        AttnOp op;
        if (!attn_prepare(op, q, Lq, k, v, Lk, a, &err))
            return bad(err);
        P.add([op](cudaStream_t s) { return attn_launch(op, s); });
    }
};

// Plans are cached per geometry key.
using PlanMap = std::map<std::vector<int>, std::unique_ptr<Plan>>;

}  // namespace

// ================================================================================================ UNet

struct UnetImpl {
    mkb_unet_config cfg{};
    int C0 = 0, TE = 0, ADD = 0;
    WTable W;
    cudaStream_t stream = nullptr;
    uint32_t* status = nullptr;
    struct Op {
        enum Kind { kConvIn, kPush, kRes, kAttn, kDown, kCat, kUp } kind;
        std::string name;
        int cin = 0, cout = 0, depth = 0, emb_off = 0, tfirst = 0;
    };
    std::vector<Op> ops;
    int emb_rows = 0, n_tblocks = 0;
    // per slot: added conditioning, context length, cross-attention K / V per transformer block [slots][H][S][64]
    float* y = nullptr;
    std::vector<int> ctx_rows;
    std::vector<__nv_bfloat16*> kc, vc;  // per transformer block
    std::vector<int> tb_c;               // channels of each transformer block
    __nv_bfloat16* ctx_bf = nullptr;
    float* ctx_f = nullptr;
    int gh = 0, gw = 0;
    PlanMap plans;
    float *tokens = nullptr, *eps_tok = nullptr, *tsin = nullptr;
    mkb_probe_fn probe = nullptr;
    void* probe_user = nullptr;

    ~UnetImpl()
    {
        plans.clear();
        W.release();
        for (void* p : {(void*)y, (void*)ctx_bf, (void*)ctx_f, (void*)tokens, (void*)eps_tok, (void*)tsin})
            if (p)
                cudaFree(p);
        for (auto* p : kc)
            cudaFree(p);
        for (auto* p : vc)
            cudaFree(p);
        if (stream)
            cudaStreamDestroy(stream);
    }

    mkb_status create(const mkb_unet_config& c);
    // The plan of B samples that use slots slot0 .. slot0 + B - 1.
    mkb_status build(int B, int slot0, Plan** out);
    // One step of the samples whose latents are in `tokens`; eps lands in `eps_tok`.
    mkb_status run_step(int B, int slot0, const float* sigmas, cudaStream_t s);
    double flops(int B) const;
};

mkb_status UnetImpl::create(const mkb_unet_config& c)
{
    cfg = c;
    C0 = c.channels[0];
    TE = 4 * C0;
    ADD = c.pooled_dim + kAdded6;
    for (int l = 0; l < 3; ++l)
        if (c.channels[l] <= 0 || c.channels[l] % 64 || c.depth[l] < 0)
            return fail(MKB_ERR_INVALID, "unet: channels must be positive multiples of 64");
    if (c.layers < 1 || c.context_dim % 8 || c.context_dim <= 0 || c.pooled_dim % 8 || c.max_batch < 1 ||
        c.max_batch > 8 || c.max_gh < 4 || c.max_gw < 4 || c.max_context < 1 || c.slots < 1 || c.depth[2] < 1)
        return fail(MKB_ERR_INVALID, "unet: bad configuration");
    // Block list, as oracle/sdxl.py's unet_structure and sdxl.cpp's input / middle / output blocks.
    int ch = C0, blk = 1;
    std::vector<int> skips;
    ops.push_back({Op::kConvIn, "conv_in", 4, C0});
    ops.push_back({Op::kPush, "", 0, C0});
    skips.push_back(C0);
    auto res = [&](const std::string& n, int cin, int cout) {
        Op o{Op::kRes, n, cin, cout};
        o.emb_off = emb_rows;
        emb_rows += cout;
        ops.push_back(o);
    };
    auto attn = [&](const std::string& n, int cc, int d) {
        Op o{Op::kAttn, n, cc, cc, d};
        o.tfirst = n_tblocks;
        for (int j = 0; j < d; ++j)
            tb_c.push_back(cc);
        n_tblocks += d;
        ops.push_back(o);
    };
    for (int l = 0; l < 3; ++l) {
        for (int k = 0; k < c.layers; ++k) {
            res("in" + std::to_string(blk) + ".res", ch, c.channels[l]);
            ch = c.channels[l];
            if (c.depth[l])
                attn("in" + std::to_string(blk) + ".attn", ch, c.depth[l]);
            ops.push_back({Op::kPush, "", 0, ch});
            skips.push_back(ch);
            ++blk;
        }
        if (l < 2) {
            ops.push_back({Op::kDown, "in" + std::to_string(blk) + ".down", ch, ch});
            ops.push_back({Op::kPush, "", 0, ch});
            skips.push_back(ch);
            ++blk;
        }
    }
    res("mid.res0", ch, ch);
    attn("mid.attn", ch, c.depth[2]);
    res("mid.res1", ch, ch);
    blk = 0;
    for (int l = 2; l >= 0; --l)
        for (int k = 0; k <= c.layers; ++k) {
            const int sc = skips.back();
            skips.pop_back();
            ops.push_back({Op::kCat, "", ch, sc});
            res("out" + std::to_string(blk) + ".res", ch + sc, c.channels[l]);
            ch = c.channels[l];
            if (c.depth[l])
                attn("out" + std::to_string(blk) + ".attn", ch, c.depth[l]);
            if (l > 0 && k == c.layers)
                ops.push_back({Op::kUp, "out" + std::to_string(blk) + ".up", ch, ch});
            ++blk;
        }
    // Weights: every residual block's time-embedding projection first, stacked for one GEMV.
    for (const Op& o : ops)
        if (o.kind == Op::kRes)
            W.add(o.name + ".emb.w", WTable::kMat, o.cout, TE);
    for (const Op& o : ops)
        if (o.kind == Op::kRes)
            W.add(o.name + ".emb.b", WTable::kVec, o.cout);
    W.add("time.lin1.w", WTable::kMat, TE, C0);
    W.add("time.lin1.b", WTable::kVec, TE);
    W.add("time.lin2.w", WTable::kMat, TE, TE);
    W.add("time.lin2.b", WTable::kVec, TE);
    W.add("label.lin1.w", WTable::kMat, TE, ADD);
    W.add("label.lin1.b", WTable::kVec, TE);
    W.add("label.lin2.w", WTable::kMat, TE, TE);
    W.add("label.lin2.b", WTable::kVec, TE);
    for (const Op& o : ops) {
        switch (o.kind) {
        case Op::kConvIn:
            W.add("conv_in.w", WTable::kConv3, o.cout, 4, 0, 64);
            W.add("conv_in.b", WTable::kVec, o.cout);
            break;
        case Op::kRes:
            W.add(o.name + ".gn1.w", WTable::kVec, o.cin, 0, 0, 0, true);
            W.add(o.name + ".gn1.b", WTable::kVec, o.cin);
            W.add(o.name + ".conv1.w", WTable::kConv3, o.cout, o.cin);
            W.add(o.name + ".conv1.b", WTable::kVec, o.cout);
            W.add(o.name + ".gn2.w", WTable::kVec, o.cout, 0, 0, 0, true);
            W.add(o.name + ".gn2.b", WTable::kVec, o.cout);
            W.add(o.name + ".conv2.w", WTable::kConv3, o.cout, o.cout);
            W.add(o.name + ".conv2.b", WTable::kVec, o.cout);
            if (o.cin != o.cout) {
                W.add(o.name + ".skip.w", WTable::kMat, o.cout, o.cin);
                W.add(o.name + ".skip.b", WTable::kVec, o.cout);
            }
            break;
        case Op::kAttn: {
            const int cc = o.cin;
            W.add(o.name + ".gn.w", WTable::kVec, cc, 0, 0, 0, true);
            W.add(o.name + ".gn.b", WTable::kVec, cc);
            W.add(o.name + ".proj_in.w", WTable::kMat, cc, cc);
            W.add(o.name + ".proj_in.b", WTable::kVec, cc);
            W.add(o.name + ".proj_out.w", WTable::kMat, cc, cc);
            W.add(o.name + ".proj_out.b", WTable::kVec, cc);
            for (int j = 0; j < o.depth; ++j) {
                const std::string p = o.name + ".b" + std::to_string(j) + ".";
                W.add(p + "ln1.w", WTable::kVec, cc, 0, 0, 0, true);
                W.add(p + "ln1.b", WTable::kVec, cc);
                W.add(p + "qkv.w", WTable::kMat, 3 * cc, cc);
                W.add(p + "o1.w", WTable::kMat, cc, cc);
                W.add(p + "o1.b", WTable::kVec, cc);
                W.add(p + "ln2.w", WTable::kVec, cc, 0, 0, 0, true);
                W.add(p + "ln2.b", WTable::kVec, cc);
                W.add(p + "q2.w", WTable::kMat, cc, cc);
                W.add(p + "kv2.w", WTable::kMat, 2 * cc, c.context_dim);
                W.add(p + "o2.w", WTable::kMat, cc, cc);
                W.add(p + "o2.b", WTable::kVec, cc);
                W.add(p + "ln3.w", WTable::kVec, cc, 0, 0, 0, true);
                W.add(p + "ln3.b", WTable::kVec, cc);
                W.add(p + "ff1.w", WTable::kGlu, 8 * cc, cc);
                W.add(p + "ff1.b", WTable::kGluVec, 8 * cc);
                W.add(p + "ff2.w", WTable::kMat, cc, 4 * cc);
                W.add(p + "ff2.b", WTable::kVec, cc);
            }
            break;
        }
        case Op::kDown:
        case Op::kUp:
            W.add(o.name + ".w", WTable::kConv3, o.cin, o.cin);
            W.add(o.name + ".b", WTable::kVec, o.cin);
            break;
        default:
            break;
        }
    }
    W.add("out.gn.w", WTable::kVec, C0, 0, 0, 0, true);
    W.add("out.gn.b", WTable::kVec, C0);
    W.add("out.conv.w", WTable::kConv3, 4, C0, 32, 0);
    W.add("out.conv.b", WTable::kVec, 4, 0, 32);
    MKB_TRY_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    status = device_status_word();
    MKB_TRY(W.alloc());
    const size_t S = c.max_context;
    MKB_TRY_CUDA(cudaMalloc(&y, size_t(c.slots) * ADD * 4), "unet");
    MKB_TRY_CUDA(cudaMalloc(&ctx_f, S * c.context_dim * 4), "unet");
    MKB_TRY_CUDA(cudaMalloc(&ctx_bf, S * c.context_dim * 2), "unet");
    MKB_TRY_CUDA(cudaMalloc(&tokens, size_t(c.max_batch) * c.max_gh * c.max_gw * 16 * 4), "unet");
    MKB_TRY_CUDA(cudaMalloc(&eps_tok, size_t(c.max_batch) * c.max_gh * c.max_gw * 16 * 4), "unet");
    MKB_TRY_CUDA(cudaMalloc(&tsin, size_t(c.max_batch) * C0 * 4), "unet");
    ctx_rows.assign(c.slots, 0);
    for (int t = 0; t < n_tblocks; ++t) {
        __nv_bfloat16 *k = nullptr, *v = nullptr;
        const size_t n = size_t(c.slots) * tb_c[t] * S;
        MKB_TRY_CUDA(cudaMalloc(&k, n * 2), "unet kv");
        MKB_TRY_CUDA(cudaMalloc(&v, n * 2), "unet kv");
        kc.push_back(k);
        vc.push_back(v);
    }
    return MKB_OK;
}

double UnetImpl::flops(int B) const
{
    double f = 0;
    long h = 2L * gh, w = 2L * gw;
    const double S = ctx_rows.empty() ? 0 : ctx_rows[0];
    for (const Op& o : ops) {
        const double P = double(h) * w;
        switch (o.kind) {
        case Op::kConvIn: f += 2 * P * o.cout * 9 * 4; break;
        case Op::kRes:
            f += 2 * P * o.cout * 9 * (o.cin + o.cout) + (o.cin != o.cout ? 2 * P * o.cout * o.cin : 0);
            break;
        case Op::kAttn: {
            const double c = o.cin;
            f += 4 * P * c * c + o.depth * (36 * P * c * c + 4 * P * P * c + 4 * P * S * c);
            break;
        }
        case Op::kDown:
            h /= 2, w /= 2;
            f += 2 * double(h) * w * o.cin * 9 * o.cin;
            break;
        case Op::kUp:
            h *= 2, w *= 2;
            f += 2 * double(h) * w * o.cin * 9 * o.cin;
            break;
        default: break;
        }
    }
    f += 2 * 4.0 * gh * gw * 4 * 9 * C0;  // conv_out
    return f * B;
}

mkb_status UnetImpl::build(int B, int slot0, Plan** out)
{
    const std::vector<int> key = {B, gh, gw, ctx_rows[slot0], slot0};
    auto it = plans.find(key);
    if (it != plans.end()) {
        *out = it->second.get();
        return MKB_OK;
    }
    auto plan = std::make_unique<Plan>();
    Plan& P = *plan;
    mkb_status st = MKB_OK;
    Builder bd{P, status};
    const int H0 = 2 * gh, W0 = 2 * gw, S = ctx_rows[slot0];
    // Buffer sizes: the widest fp32 image of any stage (channels incl. a concatenation) and the transformer's.
    size_t most = size_t(H0) * W0 * 64, tmost = 1, gnmost = 0;
    {
        long h = H0, w = W0;
        for (const Op& o : ops) {
            const size_t Pp = size_t(h) * w;
            if (o.kind == Op::kDown)
                h /= 2, w /= 2;
            if (o.kind == Op::kUp)
                h *= 2, w *= 2;
            const size_t P2 = size_t(h) * w;
            most = std::max({most, Pp * size_t(o.cin + (o.kind == Op::kCat ? o.cout : 0)), Pp * size_t(o.cout),
                             P2 * size_t(o.cout)});
            if (o.kind == Op::kAttn)
                tmost = std::max(tmost, Pp * size_t(o.cin));
            gnmost = std::max(gnmost, group_norm_workspace(B, int(Pp), std::max(o.cin, o.cout), 32));
        }
    }
    const size_t Bm = size_t(B);
    float* F[3];
    for (auto& f : F)
        f = P.buf<float>(Bm * most, &st);
    float* CAT = P.buf<float>(Bm * most, &st);
    float* U = P.buf<float>(Bm * most, &st);
    float* SK = P.buf<float>(Bm * most, &st);
    __nv_bfloat16* T = P.buf<__nv_bfloat16>(Bm * most, &st);
    __nv_bfloat16* T2 = P.buf<__nv_bfloat16>(Bm * most, &st);
    float* HS = P.buf<float>(Bm * tmost, &st);
    __nv_bfloat16* HN = P.buf<__nv_bfloat16>(Bm * tmost, &st);
    __nv_bfloat16* QH = P.buf<__nv_bfloat16>(Bm * tmost, &st);
    __nv_bfloat16* KH = P.buf<__nv_bfloat16>(Bm * tmost, &st);
    __nv_bfloat16* VH = P.buf<__nv_bfloat16>(Bm * tmost, &st);
    __nv_bfloat16* ATT = P.buf<__nv_bfloat16>(Bm * tmost, &st);
    __nv_bfloat16* FF = P.buf<__nv_bfloat16>(Bm * tmost * 4, &st);
    float* e1 = P.buf<float>(Bm * TE, &st);
    float* emb = P.buf<float>(Bm * TE, &st);
    float* l1 = P.buf<float>(Bm * TE, &st);
    float* l2 = P.buf<float>(Bm * TE, &st);
    float* se = P.buf<float>(Bm * TE, &st);
    float* eo = P.buf<float>(Bm * emb_rows, &st);
    __nv_bfloat16* lat = P.buf<__nv_bfloat16>(Bm * H0 * W0 * 64, &st);
    float* EPS = P.buf<float>(Bm * H0 * W0 * 32, &st);
    P.gn_ws = P.buf<float>(gnmost / 4 + 16, &st);
    if (st != MKB_OK)
        return st;

    // Time and label embeddings, then every residual block's projection of silu(emb) (sdxl.cpp:842-857).
    const WTable& w = W;
    const float* ty = y + size_t(slot0) * ADD;
    const float* ts = tsin;
    P.add([=, &w](cudaStream_t s) {
        return gemv(w.M("time.lin1.w"), ts, C0, w.V("time.lin1.b"), e1, TE, B, TE, C0, kActSilu, s);
    });
    P.add([=, &w](cudaStream_t s) {
        return gemv(w.M("time.lin2.w"), e1, TE, w.V("time.lin2.b"), emb, TE, B, TE, TE, kActNone, s);
    });
    P.probe("temb", -1, emb, long(B) * TE);
    const int ADDc = ADD;
    P.add([=, &w](cudaStream_t s) {
        return gemv(w.M("label.lin1.w"), ty, ADDc, w.V("label.lin1.b"), l1, TE, B, TE, ADDc, kActSilu, s);
    });
    P.add([=, &w](cudaStream_t s) {
        return gemv(w.M("label.lin2.w"), l1, TE, w.V("label.lin2.b"), l2, TE, B, TE, TE, kActNone, s);
    });
    P.add([=](cudaStream_t s) { return add_silu(emb, l2, se, size_t(B) * TE, s); });
    const int er = emb_rows;
    P.add([=, &w](cudaStream_t s) { return gemv(w.mat, se, TE, w.vec, eo, er, B, er, TE, kActNone, s); });
    float* tok = tokens;
    // conv_in's input: the tokens unpacked to [B][2gh][2gw][64] (4 channels used) and scaled (sdxl.cpp:834).
    // The scale 1 / sqrt(sigma^2 + 1) is applied on the host into the tokens buffer.
    const int ghh = gh, gww = gw;
    P.add([=](cudaStream_t s) { return unpack_tokens_bf16(tok, lat, B, ghh, gww, 64, 1.0f, s); });

    std::vector<std::pair<float*, int>> skips;  // skip tensors and their channels
    float* cur = nullptr;
    int h = H0, wd = W0, c = 4;
    auto pick = [&](const float* not1, const float* not2 = nullptr) {
        for (float* f : F)
            if (f != not1 && f != not2)
                return f;
        return F[0];
    };
    for (size_t i = 0; i < ops.size() && bd.ok(); ++i) {
        const Op& o = ops[i];
        const bool push_next = i + 1 < ops.size() && ops[i + 1].kind == Op::kPush;
        const long HW = long(h) * wd;
        float* outb = nullptr;
        if (push_next && o.kind != Op::kPush) {
            const long oh = o.kind == Op::kDown ? h / 2 : h, ow = o.kind == Op::kDown ? wd / 2 : wd;
            outb = P.buf<float>(Bm * oh * ow * o.cout, &st);
            if (st != MKB_OK)
                return st;
        }
        switch (o.kind) {
        case Op::kConvIn:
            outb = outb ? outb : pick(nullptr);
            bd.conv(lat, B, h, wd, 64, w.M("conv_in.w"), o.cout, 9, 1, w.V("conv_in.b"), nullptr, 0, nullptr, outb,
                    o.cout, true);
            cur = outb;
            c = o.cout;
            P.probe("conv_in", -1, cur, long(B) * HW * c);
            break;
        case Op::kPush:
            skips.push_back({cur, c});
            break;
        case Op::kRes: {
            // sdxl.cpp:722-740
            const float* X = cur;
            float* Y = outb ? outb : pick(X);
            bd.gn(X, T, w.V(o.name + ".gn1.w"), w.V(o.name + ".gn1.b"), B, int(HW), o.cin, 1e-5f, true);
            bd.conv(T, B, h, wd, o.cin, w.M(o.name + ".conv1.w"), o.cout, 9, 1, w.V(o.name + ".conv1.b"),
                    eo + o.emb_off, emb_rows, nullptr, U, o.cout, true);
            bd.gn(U, T, w.V(o.name + ".gn2.w"), w.V(o.name + ".gn2.b"), B, int(HW), o.cout, 1e-5f, true);
            const float* R = X;
            if (o.cin != o.cout) {
                const float* Xc = X;
                const size_t n = Bm * HW * o.cin;
                P.add([=](cudaStream_t s) { return cast_f32_bf16(Xc, T2, n, s); });
                GemmArgs a;
                a.M = int(B * HW);
                a.N = o.cout;
                a.K = o.cin;
                a.bias = w.V(o.name + ".skip.b");
                a.out = SK;
                a.ldo = o.cout;
                a.out_f32 = 1;
                bd.gemm(Epi::kAdd, T2, o.cin, w.M(o.name + ".skip.w"), o.cin, a);
                R = SK;
            }
            bd.conv(T, B, h, wd, o.cout, w.M(o.name + ".conv2.w"), o.cout, 9, 1, w.V(o.name + ".conv2.b"), nullptr,
                    0, R, Y, o.cout, true);
            cur = Y;
            c = o.cout;
            P.probe(o.name, -1, cur, long(B) * HW * c);
            break;
        }
        case Op::kAttn: {
            // sdxl.cpp:742-796
            const int cc = o.cin, heads = cc / kHead, M = int(B * HW);
            const float* X = cur;
            float* Y = outb ? outb : pick(X);
            bd.gn(X, HN, w.V(o.name + ".gn.w"), w.V(o.name + ".gn.b"), B, int(HW), cc, 1e-6f, false);
            GemmArgs pa;
            pa.M = M;
            pa.N = cc;
            pa.K = cc;
            pa.bias = w.V(o.name + ".proj_in.b");
            pa.out = HS;
            pa.ldo = cc;
            pa.out_f32 = 1;
            bd.gemm(Epi::kAdd, HN, cc, w.M(o.name + ".proj_in.w"), cc, pa);
            for (int j = 0; j < o.depth; ++j) {
                const std::string p = o.name + ".b" + std::to_string(j) + ".";
                const int tb = o.tfirst + j;
                auto ln = [&](const char* nm) {
                    LnModArgs la{};
                    la.x = HS;
                    la.y = HN;
                    la.scale = w.V(p + nm + std::string(".w"));
                    la.shift = w.V(p + nm + std::string(".b"));
                    la.rows = M;
                    la.D = cc;
                    la.rows_per_sample = M;
                    la.eps = 1e-5f;
                    la.affine = 1;
                    if (cc % 128 || cc > 4096)
                        return bd.bad("transformer width must be a multiple of 128");
                    P.add([la](cudaStream_t s) { return ln_modulate(la, s); });
                };
                ln("ln1");
                GemmArgs q;
                q.M = M;
                q.N = 3 * cc;
                q.K = cc;
                q.qh = QH;
                q.kh = KH;
                q.vh = VH;
                q.D = cc;
                q.head_dim = kHead;
                q.L = int(HW);
                q.seg_rows = int(HW);
                bd.gemm(Epi::kHeads, HN, cc, w.M(p + "qkv.w"), cc, q);
                bd.attn(QH, KH, VH, B, heads, int(HW), int(HW), ATT);
                GemmArgs r;
                r.M = M;
                r.N = cc;
                r.K = cc;
                r.bias = w.V(p + "o1.b");
                r.add_resid = HS;
                r.ld_add_resid = cc;
                r.out = HS;
                r.ldo = cc;
                r.out_f32 = 1;
                bd.gemm(Epi::kAdd, ATT, cc, w.M(p + "o1.w"), cc, r);
                ln("ln2");
                GemmArgs q2 = q;
                q2.N = cc;
                bd.gemm(Epi::kHeads, HN, cc, w.M(p + "q2.w"), cc, q2);
                const size_t kvo = size_t(slot0) * cc * S;
                bd.attn(QH, kc[tb] + kvo, vc[tb] + kvo, B, heads, int(HW), S, ATT);
                GemmArgs r2 = r;
                r2.bias = w.V(p + "o2.b");
                bd.gemm(Epi::kAdd, ATT, cc, w.M(p + "o2.w"), cc, r2);
                ln("ln3");
                GemmArgs g;
                g.M = M;
                g.N = 8 * cc;
                g.K = cc;
                g.bias = w.V(p + "ff1.b");
                g.out = FF;
                g.ldo = 4 * cc;
                g.glu = kGluGelu;
                bd.gemm(Epi::kSwiGLU, HN, cc, w.M(p + "ff1.w"), cc, g);
                GemmArgs r3 = r;
                r3.K = 4 * cc;
                r3.bias = w.V(p + "ff2.b");
                bd.gemm(Epi::kAdd, FF, 4 * cc, w.M(p + "ff2.w"), 4 * cc, r3);
            }
            {
                const float* HSc = HS;
                const size_t n = Bm * HW * cc;
                P.add([=](cudaStream_t s) { return cast_f32_bf16(HSc, HN, n, s); });
            }
            GemmArgs po;
            po.M = M;
            po.N = cc;
            po.K = cc;
            po.bias = w.V(o.name + ".proj_out.b");
            po.add_resid = X;
            po.ld_add_resid = cc;
            po.out = Y;
            po.ldo = cc;
            po.out_f32 = 1;
            bd.gemm(Epi::kAdd, HN, cc, w.M(o.name + ".proj_out.w"), cc, po);
            cur = Y;
            P.probe(o.name, -1, cur, long(B) * HW * cc);
            break;
        }
        case Op::kDown: {
            const float* X = cur;
            float* Y = outb ? outb : pick(X);
            const size_t n = Bm * HW * o.cin;
            P.add([=](cudaStream_t s) { return cast_f32_bf16(X, T, n, s); });
            bd.conv(T, B, h, wd, o.cin, w.M(o.name + ".w"), o.cin, 9, 2, w.V(o.name + ".b"), nullptr, 0, nullptr, Y,
                    o.cin, true);
            h /= 2, wd /= 2;
            cur = Y;
            P.probe(o.name, -1, cur, long(B) * h * wd * c);
            break;
        }
        case Op::kCat: {
            const auto sk = skips.back();
            skips.pop_back();
            const float* X = cur;
            const int ca = c;
            const long Pn = long(B) * HW;
            P.add([=](cudaStream_t s) { return concat_channels(X, ca, sk.first, sk.second, CAT, Pn, s); });
            cur = CAT;
            c = ca + sk.second;
            break;
        }
        case Op::kUp: {
            const float* X = cur;
            float* Y = pick(X);
            const int hh = h, ww2 = wd, cc = o.cin;
            P.add([=](cudaStream_t s) { return upsample2x_bf16(X, T, B, hh, ww2, cc, s); });
            h *= 2, wd *= 2;
            bd.conv(T, B, h, wd, o.cin, w.M(o.name + ".w"), o.cin, 9, 1, w.V(o.name + ".b"), nullptr, 0, nullptr, Y,
                    o.cin, true);
            cur = Y;
            P.probe(o.name, -1, cur, long(B) * h * wd * c);
            break;
        }
        }
    }
    if (!bd.ok())
        return bd.st;
    // GroupNorm + SiLU + conv_out (4 channels, padded to 32), eps repacked as tokens (sdxl.cpp:941-952).
    bd.gn(cur, T, w.V("out.gn.w"), w.V("out.gn.b"), B, h * wd, c, 1e-5f, true);
    bd.conv(T, B, h, wd, c, w.M("out.conv.w"), 32, 9, 1, w.V("out.conv.b"), nullptr, 0, nullptr, EPS, 32, true);
    float* et = eps_tok;
    P.add([=](cudaStream_t s) { return pack_tokens(EPS, 32, et, B, ghh, gww, s); });
    if (!bd.ok())
        return bd.st;
    *out = plan.get();
    plans[key] = std::move(plan);
    return MKB_OK;
}

// ================================================================================================ VAE

struct VaeImpl {
    mkb_vae_config cfg{};
    WTable W;
    cudaStream_t stream = nullptr;
    uint32_t* status = nullptr;
    struct Op {
        enum Kind { kRes, kAttn, kUp } kind;
        std::string name;
        int cin, cout;
    };
    std::vector<Op> ops;  // after conv_in
    int ctop = 0;
    int z = 4;                    // latent channels; a token holds 4 z values (2x2 patches)
    float* lat_aff = nullptr;     // per token value: [4 z] multipliers, then [4 z] offsets (latent statistics)
    PlanMap plans;
    float *tokens = nullptr, *rgba = nullptr;
    mkb_probe_fn probe = nullptr;
    void* probe_user = nullptr;

    ~VaeImpl()
    {
        plans.clear();
        W.release();
        if (tokens)
            cudaFree(tokens);
        if (rgba)
            cudaFree(rgba);
        if (lat_aff)
            cudaFree(lat_aff);
        if (stream)
            cudaStreamDestroy(stream);
    }
    mkb_status create(const mkb_vae_config& c);
    mkb_status build(int gh, int gw, Plan** out);
    double flops(int gh, int gw) const;
};

mkb_status VaeImpl::create(const mkb_vae_config& c)
{
    cfg = c;
    for (int l = 0; l < 4; ++l)
        if (c.channels[l] <= 0 || c.channels[l] % 128)
            return fail(MKB_ERR_INVALID, "vae: channels must be positive multiples of 128");
    if (c.layers < 1 || (c.latent != 4 && c.latent != 16) || !(c.scale > 0) || c.max_gh < 1 || c.max_gw < 1)
        return fail(MKB_ERR_INVALID, "vae: bad configuration (4 or 16 latent channels)");
    z = c.latent;
    ctop = c.channels[3];
    int ch = ctop;
    ops.push_back({Op::kRes, "mid.res0", ch, ch});
    ops.push_back({Op::kAttn, "mid.attn", ch, ch});
    ops.push_back({Op::kRes, "mid.res1", ch, ch});
    for (int i = 0; i < 4; ++i) {
        const int lvl = 3 - i;
        for (int k = 0; k <= c.layers; ++k) {
            ops.push_back({Op::kRes, "up" + std::to_string(i) + ".res" + std::to_string(k), ch, c.channels[lvl]});
            ch = c.channels[lvl];
        }
        if (i < 3)
            ops.push_back({Op::kUp, "up" + std::to_string(i) + ".up", ch, ch});
    }
    W.add("post_quant.w", WTable::kMat, z, z, 64, 64);
    W.add("post_quant.b", WTable::kVec, z, 0, 64);
    W.add("conv_in.w", WTable::kConv3, ctop, z, 0, 64);
    W.add("conv_in.b", WTable::kVec, ctop);
    for (const Op& o : ops) {
        if (o.kind == Op::kRes) {
            W.add(o.name + ".gn1.w", WTable::kVec, o.cin, 0, 0, 0, true);
            W.add(o.name + ".gn1.b", WTable::kVec, o.cin);
            W.add(o.name + ".conv1.w", WTable::kConv3, o.cout, o.cin);
            W.add(o.name + ".conv1.b", WTable::kVec, o.cout);
            W.add(o.name + ".gn2.w", WTable::kVec, o.cout, 0, 0, 0, true);
            W.add(o.name + ".gn2.b", WTable::kVec, o.cout);
            W.add(o.name + ".conv2.w", WTable::kConv3, o.cout, o.cout);
            W.add(o.name + ".conv2.b", WTable::kVec, o.cout);
            if (o.cin != o.cout) {
                W.add(o.name + ".skip.w", WTable::kMat, o.cout, o.cin);
                W.add(o.name + ".skip.b", WTable::kVec, o.cout);
            }
        } else if (o.kind == Op::kAttn) {
            W.add("mid.attn.gn.w", WTable::kVec, o.cin, 0, 0, 0, true);
            W.add("mid.attn.gn.b", WTable::kVec, o.cin);
            W.add("mid.attn.qkv.w", WTable::kMat, 3 * o.cin, o.cin);
            W.add("mid.attn.qkv.b", WTable::kVec, 3 * o.cin);
            W.add("mid.attn.proj.w", WTable::kMat, o.cin, o.cin);
            W.add("mid.attn.proj.b", WTable::kVec, o.cin);
        } else {
            W.add(o.name + ".w", WTable::kConv3, o.cin, o.cin);
            W.add(o.name + ".b", WTable::kVec, o.cin);
        }
    }
    W.add("out.gn.w", WTable::kVec, c.channels[0], 0, 0, 0, true);
    W.add("out.gn.b", WTable::kVec, c.channels[0]);
    W.add("out.conv.w", WTable::kConv3, 3, c.channels[0], 32, 0);
    W.add("out.conv.b", WTable::kVec, 3, 0, 32);
    MKB_TRY_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    status = device_status_word();
    MKB_TRY(W.alloc());
    MKB_TRY_CUDA(cudaMalloc(&tokens, size_t(c.max_gh) * c.max_gw * 4 * z * 4), "vae");
    MKB_TRY_CUDA(cudaMalloc(&rgba, size_t(c.max_gh) * c.max_gw * 256 * 4 * 4), "vae");
    // Latent statistics: by default tokens / scale (mean 0, deviation 1 / scale for every value).
    std::vector<float> aff(8 * z, 0.0f);
    std::fill(aff.begin(), aff.begin() + 4 * z, 1.0f / c.scale);
    MKB_TRY_CUDA(cudaMalloc(&lat_aff, aff.size() * 4), "vae");
    MKB_TRY_CUDA(cudaMemcpy(lat_aff, aff.data(), aff.size() * 4, cudaMemcpyHostToDevice), "vae");
    return MKB_OK;
}

double VaeImpl::flops(int gh, int gw) const
{
    double h = 2.0 * gh, w = 2.0 * gw;
    double f = 2 * h * w * ctop * 9 * z;
    for (const Op& o : ops) {
        const double P = h * w;
        if (o.kind == Op::kRes)
            f += 2 * P * o.cout * 9 * (o.cin + o.cout) + (o.cin != o.cout ? 2 * P * o.cout * o.cin : 0);
        else if (o.kind == Op::kAttn)
            f += 2 * P * o.cin * 4 * o.cin + 4 * P * P * o.cin;
        else {
            h *= 2, w *= 2;
            f += 2 * h * w * o.cin * 9 * o.cin;
        }
    }
    return f + 2 * h * w * 3 * 9 * cfg.channels[0];
}

mkb_status VaeImpl::build(int gh, int gw, Plan** out)
{
    const std::vector<int> key = {gh, gw};
    auto it = plans.find(key);
    if (it != plans.end()) {
        *out = it->second.get();
        return MKB_OK;
    }
    auto plan = std::make_unique<Plan>();
    Plan& P = *plan;
    mkb_status st = MKB_OK;
    Builder bd{P, status};
    const int H0 = 2 * gh, W0 = 2 * gw;
    size_t most = size_t(H0) * W0 * ctop, gnmost = 0;
    {
        size_t h = H0, w = W0;
        for (const Op& o : ops) {
            most = std::max(most, h * w * size_t(std::max(o.cin, o.cout)));
            gnmost = std::max(gnmost, group_norm_workspace(1, int(h * w), std::max(o.cin, o.cout), 32));
            if (o.kind == Op::kUp) {
                h *= 2, w *= 2;
                most = std::max(most, h * w * size_t(o.cout));
                gnmost = std::max(gnmost, group_norm_workspace(1, int(h * w), o.cout, 32));
            }
        }
        most = std::max(most, h * w * 32);
    }
    float* F[3];
    for (auto& f : F)
        f = P.buf<float>(most, &st);
    float* U = P.buf<float>(most, &st);
    float* SK = P.buf<float>(most, &st);
    __nv_bfloat16* T = P.buf<__nv_bfloat16>(most, &st);
    __nv_bfloat16* T2 = P.buf<__nv_bfloat16>(most, &st);
    __nv_bfloat16* LAT = P.buf<__nv_bfloat16>(size_t(H0) * W0 * 64, &st);
    __nv_bfloat16* PQ = P.buf<__nv_bfloat16>(size_t(H0) * W0 * 64, &st);
    const int n = H0 * W0, ca = ctop;
    // mid attention: q/k/v rows; one flash kernel at 256 / 512 channels, else V^T and the score chunk (queries per
    // pass so scores stay near 256 MB) for score GEMMs, a row softmax and P V GEMMs
    const bool flash = vae_flash_enabled() && (ca == 256 || ca == 512);
    const int qn = std::min(n, std::max(128, int((size_t(64) << 20) / size_t(n)) / 128 * 128));
    __nv_bfloat16* QKV = P.buf<__nv_bfloat16>(size_t(n) * 3 * ca, &st);
    __nv_bfloat16* VT = flash ? nullptr : P.buf<__nv_bfloat16>(size_t(n) * ca, &st);
    float* SC = flash ? nullptr : P.buf<float>(size_t(qn) * n, &st);
    __nv_bfloat16* PR = flash ? nullptr : P.buf<__nv_bfloat16>(size_t(qn) * n, &st);
    __nv_bfloat16* AT = P.buf<__nv_bfloat16>(size_t(n) * ca, &st);
    P.gn_ws = P.buf<float>(std::max(gnmost / 4, size_t(32) * 128) + 16, &st);  // also the fused path's segments
    // GroupNorm statistics left by the convolutions (where every channel count of the decoder gives groups of 4, 8
    // or 16): GA for the residual stream (conv_in, each block's conv2, the upsampling convolutions), GB for conv1.
    const bool fuse = gn_fused_enabled();
    size_t parts_most = 0;
    {
        int hh = H0, ww = W0;
        for (const Op& o : ops)
            if (o.kind == Op::kUp)
                hh *= 2, ww *= 2;
        parts_most = size_t(conv_gn_chunks(hh, ww)) * 32;
    }
    float4* GA = fuse ? P.buf<float4>(parts_most, &st) : nullptr;
    float4* GB = fuse ? P.buf<float4>(parts_most, &st) : nullptr;
    if (st != MKB_OK)
        return st;
    const WTable& w = W;
    // Latents (tokens times the latent deviation plus the mean, unpacked), post_quant 1x1 (z -> z, padded to 64 both
    // ways), conv_in.
    float* tok = tokens;
    const float* aff = lat_aff;
    const int zz = z;
    P.add([=](cudaStream_t s) { return unpack_tokens_affine_bf16(tok, LAT, gh, gw, zz, 64, aff, s); });
    {
        GemmArgs a;
        a.M = n;
        a.N = 64;
        a.K = 64;
        a.bias = w.V("post_quant.b");
        a.out = PQ;
        a.ldo = 64;
        a.out_f32 = 0;
        bd.gemm(Epi::kAdd, LAT, 64, w.M("post_quant.w"), 64, a, 64);
    }
    float* cur = F[0];
    // Whether cur's statistics are in GA (it came from a convolution whose channels split into groups of 4..16).
    auto can_fuse = [&](int C) { return fuse && C % 32 == 0 && (C / 32 == 4 || C / 32 == 8 || C / 32 == 16); };
    bool cur_parts = can_fuse(ctop);
    bd.conv(PQ, 1, H0, W0, 64, w.M("conv_in.w"), ctop, 9, 1, w.V("conv_in.b"), nullptr, 0, nullptr, cur, ctop, true,
            cur_parts ? GA : nullptr);
    P.probe("conv_in", -1, cur, long(n) * ctop);
    int h = H0, wd = W0, c = ctop;
    // GroupNorm of cur (or of conv1's output U, from GB), from the statistics when there are some.
    auto norm = [&](const float* X, bool parts, const float4* G, const std::string& wn, int C, bool silu) {
        if (parts)
            bd.gn_from(X, G, conv_gn_chunks(h, wd), T, w.V(wn + ".w"), w.V(wn + ".b"), 1, h * wd, C, 1e-6f, silu);
        else
            bd.gn(X, T, w.V(wn + ".w"), w.V(wn + ".b"), 1, h * wd, C, 1e-6f, silu);
    };
    auto pick = [&](const float* x) {
        for (float* f : F)
            if (f != x)
                return f;
        return F[0];
    };
    for (const Op& o : ops) {
        if (!bd.ok())
            break;
        const int HW = h * wd;
        if (o.kind == Op::kRes) {
            // engine.cpp:732-746 (GroupNorm eps 1e-6 in the AutoencoderKL layout)
            const float* X = cur;
            float* Y = pick(X);
            norm(X, cur_parts, GA, o.name + ".gn1", o.cin, true);
            const bool u_parts = can_fuse(o.cout);
            bd.conv(T, 1, h, wd, o.cin, w.M(o.name + ".conv1.w"), o.cout, 9, 1, w.V(o.name + ".conv1.b"), nullptr, 0,
                    nullptr, U, o.cout, true, u_parts ? GB : nullptr);
            norm(U, u_parts, GB, o.name + ".gn2", o.cout, true);
            const float* R = X;
            if (o.cin != o.cout) {
                const size_t cnt = size_t(HW) * o.cin;
                P.add([=](cudaStream_t s) { return cast_f32_bf16(X, T2, cnt, s); });
                GemmArgs a;
                a.M = HW;
                a.N = o.cout;
                a.K = o.cin;
                a.bias = w.V(o.name + ".skip.b");
                a.out = SK;
                a.ldo = o.cout;
                a.out_f32 = 1;
                bd.gemm(Epi::kAdd, T2, o.cin, w.M(o.name + ".skip.w"), o.cin, a);
                R = SK;
            }
            cur_parts = can_fuse(o.cout);
            bd.conv(T, 1, h, wd, o.cout, w.M(o.name + ".conv2.w"), o.cout, 9, 1, w.V(o.name + ".conv2.b"), nullptr,
                    0, R, Y, o.cout, true, cur_parts ? GA : nullptr);
            cur = Y;
            c = o.cout;
        } else if (o.kind == Op::kAttn) {
            // engine.cpp:748-778: GroupNorm, qkv 1x1, scores per query chunk, row softmax, P V, proj + residual.
            const float* X = cur;
            float* Y = pick(X);
            norm(X, cur_parts, GA, "mid.attn.gn", c, false);
            GemmArgs q;
            q.M = HW;
            q.N = 3 * c;
            q.K = c;
            q.bias = w.V("mid.attn.qkv.b");
            q.out = QKV;
            q.ldo = 3 * c;
            q.out_f32 = 0;
            bd.gemm(Epi::kAdd, T, c, w.M("mid.attn.qkv.w"), c, q);
            const int cc = c;
            const float sc = 1.0f / std::sqrt(float(c));
            if (flash) {
                AttnWideArgs wa;
                wa.n = HW;
                wa.d = c;
                wa.q_col = 0;
                wa.k_col = c;
                wa.v_col = 2 * c;
                wa.out = AT;
                wa.ldo = c;
                wa.scale_log2 = 1.4426950408889634f * sc;
                wa.status = status;
                AttnWideOp aop;
                const char* aerr = nullptr;
                if (!attn_wide_prepare(aop, QKV, 3L * c, wa, &aerr))
                    return fail(MKB_ERR_INVALID, std::string("vae plan: ") + (aerr ? aerr : "mid attention"));
                P.add([aop](cudaStream_t s) { return attn_wide_launch(aop, s); });
            } else {
                P.add([=](cudaStream_t s) { return transpose_bf16(QKV, 3L * cc, 2 * cc, VT, HW, cc, s); });
            }
            for (int q0 = 0; q0 < HW && bd.ok() && !flash; q0 += qn) {
                const int m = std::min(qn, HW - q0);
                GemmArgs sa;
                sa.M = m;
                sa.N = HW;
                sa.K = c;
                sa.out = SC;
                sa.ldo = HW;
                bd.gemm(Epi::kF32, QKV + size_t(q0) * 3 * c, 3 * c, QKV + c, 3 * c, sa);
                const int nn = HW;
                P.add([=](cudaStream_t s) { return softmax_rows_bf16(SC, PR, m, nn, sc, s); });
                GemmArgs pv;
                pv.M = m;
                pv.N = c;
                pv.K = HW;
                pv.out = AT + size_t(q0) * c;
                pv.ldo = c;
                bd.gemm(Epi::kBF16, PR, HW, VT, HW, pv);
            }
            GemmArgs pr;
            pr.M = HW;
            pr.N = c;
            pr.K = c;
            pr.bias = w.V("mid.attn.proj.b");
            pr.add_resid = X;
            pr.ld_add_resid = c;
            pr.out = Y;
            pr.ldo = c;
            pr.out_f32 = 1;
            bd.gemm(Epi::kAdd, AT, c, w.M("mid.attn.proj.w"), c, pr);
            cur = Y;
            cur_parts = false;  // a plain GEMM wrote it
        } else {
            const float* X = cur;
            float* Y = pick(X);
            const int hh = h, ww2 = wd, cc = o.cin;
            P.add([=](cudaStream_t s) { return upsample2x_bf16(X, T, 1, hh, ww2, cc, s); });
            h *= 2, wd *= 2;
            cur_parts = can_fuse(o.cin);
            bd.conv(T, 1, h, wd, o.cin, w.M(o.name + ".w"), o.cin, 9, 1, w.V(o.name + ".b"), nullptr, 0, nullptr, Y,
                    o.cin, true, cur_parts ? GA : nullptr);
            cur = Y;
        }
        P.probe(o.name, -1, cur, long(h) * wd * c);
    }
    if (!bd.ok())
        return bd.st;
    norm(cur, cur_parts, GA, "out.gn", c, true);
    float* O = pick(cur);
    bd.conv(T, 1, h, wd, c, w.M("out.conv.w"), 32, 9, 1, w.V("out.conv.b"), nullptr, 0, nullptr, O, 32, true);
    float* rg = rgba;
    const long Pn = long(h) * wd;
    P.add([=](cudaStream_t s) { return to_rgba(O, 32, rg, Pn, s); });
    if (!bd.ok())
        return bd.st;
    *out = plan.get();
    plans[key] = std::move(plan);
    return MKB_OK;
}

// ------------------------------------------------------------------------------------------------ text encoders

constexpr int kClipTokens = 77, kClipPooled = 1280, kClipEnd = 49407;
constexpr float kClipEps = 1e-5f;

// One of SDXL's text encoders (Sdxl::encode_clip, sdxl.cpp:459-546): CLIP ViT-L (which 0: quick GELU, its output the
// second to last layer's states) or OpenCLIP bigG (which 1: erf GELU, also the pooled state). Each layer: LayerNorm,
// q | k | v projection into heads of 64, causal attention over the 77 tokens, output projection added to the
// residual, LayerNorm, fc1 with the activation, fc2 added to the residual. Every projection whose input the reference
// splits into bf16 parts (docs/architecture.md:9-11) takes it as [hi | lo] against its weights held twice along K:
// the LayerNorm outputs and fc1's output. The attention output feeds the output projection as bf16.
struct ClipImpl {
    mkb_clip_config cfg{};
    WTable W;
    cudaStream_t stream = nullptr;
    uint32_t* status = nullptr;
    PlanMap plans;
    int* ids = nullptr;       // [max_chunks * 77]
    int* eos = nullptr;       // [max_chunks]: each chunk's first end token
    float* hidden = nullptr;  // [max_chunks * 77][E]
    float* pooled = nullptr;  // [max_chunks][1280]
    mkb_probe_fn probe = nullptr;
    void* probe_user = nullptr;
    std::vector<float> empty_hidden;  // the empty prompt's hidden states (computed on first need)

    ~ClipImpl()
    {
        plans.clear();
        W.release();
        for (void* p : {static_cast<void*>(ids), static_cast<void*>(eos), static_cast<void*>(hidden),
                        static_cast<void*>(pooled)})
            if (p)
                cudaFree(p);
        if (stream)
            cudaStreamDestroy(stream);
    }
    int run_layers() const { return cfg.which == 1 ? cfg.layers : cfg.layers - 1; }
    mkb_status create(const mkb_clip_config& c);
    mkb_status build(int B, Plan** out);
    mkb_status encode(const int32_t* host_ids, int B, float* hidden_out, float* pooled_out);
};

mkb_status ClipImpl::create(const mkb_clip_config& c)
{
    cfg = c;
    if ((c.which != 0 && c.which != 1) || c.width <= 0 || c.width % 128 || c.width > 2048 || c.heads * kHead != c.width ||
        c.layers < 2 || c.ffn <= 0 || c.ffn % 128 || c.vocab <= kClipEnd || c.max_chunks < 1)
        return fail(MKB_ERR_INVALID, "clip: bad configuration (width a multiple of 128 up to 2048 in heads of 64, "
                                     "ffn a multiple of 128, at least 2 layers, the CLIP vocabulary)");
    const long E = c.width, F = c.ffn;
    W.add("tok", WTable::kTab, c.vocab, E);
    W.add("pos", WTable::kTab, kClipTokens, E);
    for (int i = 0; i < c.layers; ++i) {
        const std::string p = "l" + std::to_string(i) + ".";
        W.add(p + "ln1.w", WTable::kVec, E, 0, 0, 0, true);
        W.add(p + "ln1.b", WTable::kVec, E);
        W.add(p + "qkv.w", WTable::kMatDup, 3 * E, E);
        W.add(p + "qkv.b", WTable::kVec, 3 * E);
        W.add(p + "o.w", WTable::kMat, E, E);
        W.add(p + "o.b", WTable::kVec, E);
        W.add(p + "ln2.w", WTable::kVec, E, 0, 0, 0, true);
        W.add(p + "ln2.b", WTable::kVec, E);
        W.add(p + "fc1.w", WTable::kMatDup, F, E);
        W.add(p + "fc1.b", WTable::kVec, F);
        W.add(p + "fc2.w", WTable::kMatDup, E, F);
        W.add(p + "fc2.b", WTable::kVec, E);
    }
    if (c.which == 1) {
        W.add("lnf.w", WTable::kVec, E, 0, 0, 0, true);
        W.add("lnf.b", WTable::kVec, E);
        W.add("proj", WTable::kTab, E, kClipPooled);
    }
    MKB_TRY_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    status = device_status_word();
    const size_t rows = size_t(c.max_chunks) * kClipTokens;
    MKB_TRY(W.alloc());
    MKB_TRY_CUDA(cudaMalloc(&ids, rows * 4), "clip buffers");
    MKB_TRY_CUDA(cudaMalloc(&eos, size_t(c.max_chunks) * 4), "clip buffers");
    MKB_TRY_CUDA(cudaMalloc(&hidden, rows * E * 4), "clip buffers");
    MKB_TRY_CUDA(cudaMalloc(&pooled, size_t(c.max_chunks) * kClipPooled * 4), "clip buffers");
    return MKB_OK;
}

mkb_status ClipImpl::build(int B, Plan** out)
{
    const std::vector<int> key = {B};
    auto it = plans.find(key);
    if (it != plans.end()) {
        *out = it->second.get();
        return MKB_OK;
    }
    auto plan = std::make_unique<Plan>();
    Plan& P = *plan;
    mkb_status st = MKB_OK;
    Builder bd{P, status};
    const int E = cfg.width, F = cfg.ffn, H = cfg.heads, T = kClipTokens, M = B * T;
    float* X = P.buf<float>(size_t(M) * E, &st);
    __nv_bfloat16* XS = P.buf<__nv_bfloat16>(size_t(M) * 2 * E, &st);
    __nv_bfloat16* QH = P.buf<__nv_bfloat16>(size_t(M) * E, &st);
    __nv_bfloat16* KH = P.buf<__nv_bfloat16>(size_t(M) * E, &st);
    __nv_bfloat16* VH = P.buf<__nv_bfloat16>(size_t(M) * E, &st);
    __nv_bfloat16* AT = P.buf<__nv_bfloat16>(size_t(M) * E, &st);
    float* HF = P.buf<float>(size_t(M) * F, &st);
    __nv_bfloat16* HS = P.buf<__nv_bfloat16>(size_t(M) * 2 * F, &st);
    if (st != MKB_OK)
        return st;
    const WTable& w = W;
    const int* id = ids;
    const float *tok = w.V("tok"), *pos = w.V("pos");
    P.add([=](cudaStream_t s) { return clip_embed(id, tok, pos, X, M, T, E, s); });
    AttnArgs at;  // causal over each chunk's 77 tokens: the condition-causal mask with every row a condition row
    at.B = B;
    at.H = H;
    at.Lq = T;
    at.Lk = T;
    at.mask = kMaskCondCausal;
    at.cond_len = T;
    at.head_dim = kHead;
    at.scale_log2 = 1.4426950408889634f / std::sqrt(float(kHead));
    at.split = 0;
    at.out1 = AT;
    at.ld1 = E;
    at.rows1 = T;
    at.status = status;
    AttnOp aop;
    const char* err = nullptr;
    if (!attn_prepare(aop, QH, T, KH, VH, T, at, &err))
        return fail(MKB_ERR_INVALID, std::string("clip plan: ") + (err ? err : "attention"));
    const int act = cfg.which == 0 ? kActQuickGelu : kActGeluErf;
    for (int i = 0; i < run_layers() && bd.ok(); ++i) {
        const std::string p = "l" + std::to_string(i) + ".";
        const float *g1 = w.V(p + "ln1.w"), *b1 = w.V(p + "ln1.b"), *g2 = w.V(p + "ln2.w"), *b2 = w.V(p + "ln2.b");
        P.add([=](cudaStream_t s) { return ln_split_bf16(X, g1, b1, XS, M, E, kClipEps, s); });
        GemmArgs q;
        q.M = M;
        q.N = 3 * E;
        q.K = 2 * E;
        q.bias = w.V(p + "qkv.b");
        q.qh = QH;
        q.kh = KH;
        q.vh = VH;
        q.D = E;
        q.head_dim = kHead;
        q.L = T;
        q.seg_rows = T;
        bd.gemm(Epi::kHeads, XS, 2 * E, w.M(p + "qkv.w"), 2 * E, q);
        P.add([aop](cudaStream_t s) { return attn_launch(aop, s); });
        GemmArgs o;
        o.M = M;
        o.N = E;
        o.K = E;
        o.bias = w.V(p + "o.b");
        o.add_resid = X;
        o.ld_add_resid = E;
        o.out = X;
        o.ldo = E;
        o.out_f32 = 1;
        bd.gemm(Epi::kAdd, AT, E, w.M(p + "o.w"), E, o);
        P.add([=](cudaStream_t s) { return ln_split_bf16(X, g2, b2, XS, M, E, kClipEps, s); });
        GemmArgs f1;
        f1.M = M;
        f1.N = F;
        f1.K = 2 * E;
        f1.bias = w.V(p + "fc1.b");
        f1.act = act;
        f1.out = HF;
        f1.ldo = F;
        bd.gemm(Epi::kF32, XS, 2 * E, w.M(p + "fc1.w"), 2 * E, f1);
        P.add([=](cudaStream_t s) { return split_bf16(HF, HS, M, F, s); });
        GemmArgs f2 = o;
        f2.K = 2 * F;
        f2.bias = w.V(p + "fc2.b");
        bd.gemm(Epi::kAdd, HS, 2 * F, w.M(p + "fc2.w"), 2 * F, f2);
        P.probe("layer", i, X, long(M) * E);
        if (i + 2 == cfg.layers) {
            float* hid = hidden;
            P.add([=](cudaStream_t s) {
                return cudaMemcpyAsync(hid, X, size_t(M) * E * 4, cudaMemcpyDeviceToDevice, s);
            });
        }
    }
    if (!bd.ok())
        return bd.st;
    if (cfg.which == 1) {
        const float *g = w.V("lnf.w"), *b = w.V("lnf.b"), *pr = w.V("proj");
        const int* e = eos;
        float* po = pooled;
        P.add([=](cudaStream_t s) { return clip_pooled(X, e, g, b, pr, po, B, T, E, kClipPooled, kClipEps, s); });
    }
    *out = plan.get();
    plans[key] = std::move(plan);
    return MKB_OK;
}

// Chunks of 77 ids on the host -> hidden states [B * 77][E] and (bigG) pooled states [B][1280] on the host.
mkb_status ClipImpl::encode(const int32_t* host_ids, int B, float* hidden_out, float* pooled_out)
{
    if (!host_ids || !hidden_out || B < 1 || B > cfg.max_chunks)
        return fail(MKB_ERR_INVALID, "clip_encode: null argument or chunk count out of range");
    std::vector<int> e(B, -1);
    for (int b = 0; b < B; ++b)
        for (int t = 0; t < kClipTokens; ++t) {
            const int32_t v = host_ids[size_t(b) * kClipTokens + t];
            if (v < 0 || v >= cfg.vocab)
                return fail(MKB_ERR_INVALID, "clip_encode: token out of range");
            if (v == kClipEnd && e[b] < 0)
                e[b] = t;
        }
    if (cfg.which == 1)
        for (int b = 0; b < B; ++b)
            if (e[b] < 0)
                return fail(MKB_ERR_INVALID, "clip_encode: a chunk without its end token");
    Plan* plan = nullptr;
    MKB_TRY(build(B, &plan));
    const size_t rows = size_t(B) * kClipTokens;
    MKB_TRY_CUDA(cudaMemcpyAsync(ids, host_ids, rows * 4, cudaMemcpyHostToDevice, stream), "ids upload");
    MKB_TRY_CUDA(cudaMemcpyAsync(eos, e.data(), size_t(B) * 4, cudaMemcpyHostToDevice, stream), "ids upload");
    MKB_TRY(plan->run(stream, probe, probe_user));
    MKB_TRY_CUDA(cudaMemcpyAsync(hidden_out, hidden, rows * cfg.width * 4, cudaMemcpyDeviceToHost, stream),
                 "hidden download");
    if (pooled_out && cfg.which == 1)
        MKB_TRY_CUDA(cudaMemcpyAsync(pooled_out, pooled, size_t(B) * kClipPooled * 4, cudaMemcpyDeviceToHost, stream),
                     "pooled download");
    MKB_TRY_CUDA(cudaStreamSynchronize(stream), "encode sync");
    uint32_t bits = 0;
    MKB_TRY_CUDA(cudaMemcpy(&bits, status, 4, cudaMemcpyDeviceToHost), "status");
    if (bits) {
        cudaMemset(status, 0, 4);
        return fail(MKB_ERR_KERNEL, "clip_encode: kernel status " + std::to_string(bits));
    }
    return MKB_OK;
}

namespace {

// Sdxl's discrete schedule and its timestep pick (sdxl.cpp:130-139, 643-651, 653-670).
struct SdxlSchedule {
    float sigma[1000], log_sigma[1000];
    SdxlSchedule()
    {
        double cum = 1.0;
        const double b0 = std::sqrt(0.00085), b1 = std::sqrt(0.012);
        for (int i = 0; i < 1000; ++i) {
            const double b = b0 + (b1 - b0) * double(i) / 999.0;
            cum *= 1.0 - b * b;
            const double s = std::sqrt((1.0 - cum) / cum);
            sigma[i] = float(s);
            log_sigma[i] = float(std::log(s));
        }
    }
    int timestep(float sg) const
    {
        const float ls = std::log(sg);
        int best = 0;
        for (int i = 1; i < 1000; ++i)
            if (std::abs(ls - log_sigma[i]) < std::abs(ls - log_sigma[best]))
                best = i;
        return best;
    }
};

const SdxlSchedule& sdxl_schedule()
{
    static const SdxlSchedule s;
    return s;
}

void sinusoid_host(float v, int dim, float* out)
{
    const int half = dim / 2;
    for (int i = 0; i < half; ++i) {
        const float f = std::exp(-std::log(10000.0f) * float(i) / float(half));
        out[i] = std::cos(v * f);
        out[half + i] = std::sin(v * f);
    }
}

}  // namespace

}  // namespace mkb

struct mkb_unet {
    mkb::UnetImpl impl;
};
struct mkb_vae {
    mkb::VaeImpl impl;
};

struct mkb_clip {
    mkb::ClipImpl impl;
};

using namespace mkb;

extern "C" {

mkb_status mkb_unet_create(const mkb_unet_config* cfg, mkb_unet** out)
{
    if (!cfg || !out)
        return fail(MKB_ERR_INVALID, "unet_create: null argument");
    auto* u = new (std::nothrow) mkb_unet;
    if (!u)
        return fail(MKB_ERR_ALLOC, "unet_create: host allocation");
    mkb_status s = u->impl.create(*cfg);
    if (s != MKB_OK) {
        delete u;
        return s;
    }
    *out = u;
    return MKB_OK;
}

void mkb_unet_destroy(mkb_unet* u)
{
    if (u) {
        cudaStreamSynchronize(u->impl.stream);
        delete u;
    }
}

mkb_status mkb_unet_init_random(mkb_unet* u, uint64_t seed, float std)
{
    if (!u)
        return fail(MKB_ERR_INVALID, "unet: null handle");
    return u->impl.W.init_random(seed, std, u->impl.stream);
}

int mkb_unet_weight_count(const mkb_unet* u) { return u ? int(u->impl.W.ws.size()) : 0; }

mkb_status mkb_unet_weight_lora_rows(mkb_unet* u, const char* name, long row0, long rows, const float* A,
                                     const float* B, int rank, float scale)
{
    if (!u || !name)
        return fail(MKB_ERR_INVALID, "unet lora: null argument");
    WTable& W = u->impl.W;
    const WTable::W* w = W.find(name);
    if (!w || (w->kind != WTable::kMat && w->kind != WTable::kGlu))
        return fail(MKB_ERR_INVALID, std::string("unet lora: ") + name + " is not a matrix");
    if (row0 < 0 || rows <= 0 || row0 + rows > w->r)
        return fail(MKB_ERR_INVALID, std::string("unet lora: rows out of range for ") + name);
    return lora_merge_rows(W.mat + w->off, w->cp, row0, rows, w->c, w->kind == WTable::kGlu ? w->r / 2 : 0, A, B,
                           rank, scale, u->impl.stream);
}

mkb_status mkb_unet_weight_info(const mkb_unet* u, int i, const char** name, long* dims, int* ndim)
{
    if (!u)
        return fail(MKB_ERR_INVALID, "unet: null handle");
    return u->impl.W.info(i, name, dims, ndim);
}

mkb_status mkb_unet_weight_read(mkb_unet* u, const char* name, float* host)
{
    if (!u || !name)
        return fail(MKB_ERR_INVALID, "unet: null argument");
    MKB_TRY_CUDA(cudaStreamSynchronize(u->impl.stream), "sync");
    return u->impl.W.read(name, host);
}

mkb_status mkb_unet_weight_write(mkb_unet* u, const char* name, const float* host)
{
    if (!u || !name)
        return fail(MKB_ERR_INVALID, "unet: null argument");
    MKB_TRY_CUDA(cudaStreamSynchronize(u->impl.stream), "sync");
    return u->impl.W.write(name, host);
}

mkb_status mkb_unet_begin(mkb_unet* u, const float* context, int S, const float* pooled, int gh, int gw, int slot)
{
    if (!u || !context || !pooled)
        return fail(MKB_ERR_INVALID, "unet_begin: null argument");
    UnetImpl& m = u->impl;
    if (slot < 0 || slot >= m.cfg.slots || S < 1 || S > m.cfg.max_context || gh < 4 || gw < 4 ||
        gh > m.cfg.max_gh || gw > m.cfg.max_gw || gh % 2 || gw % 16)
        return fail(MKB_ERR_INVALID, "unet_begin: slot, context rows or grid out of range (gh even, gw a multiple "
                                     "of 16 so the smallest level is 8 wide)");
    for (int s2 = 0; s2 < m.cfg.slots; ++s2)
        if (s2 != slot && m.ctx_rows[s2] && m.ctx_rows[s2] != S)
            return fail(MKB_ERR_INVALID, "unet_begin: every slot needs the same context length");
    cudaStream_t s = m.stream;
    // The added conditioning: pooled state, then (H, W, 0, 0, H, W) sinusoids (sdxl.cpp:683-692).
    std::vector<float> yv(m.ADD);
    std::copy(pooled, pooled + m.cfg.pooled_dim, yv.begin());
    const float H = float(16 * gh), W = float(16 * gw);
    const float sizes[6] = {H, W, 0.0f, 0.0f, H, W};
    for (int i = 0; i < 6; ++i)
        sinusoid_host(sizes[i], kTime, yv.data() + m.cfg.pooled_dim + i * kTime);
    MKB_TRY_CUDA(cudaMemcpyAsync(m.y + size_t(slot) * m.ADD, yv.data(), yv.size() * 4, cudaMemcpyHostToDevice, s),
                 "y upload");
    MKB_TRY_CUDA(cudaMemcpyAsync(m.ctx_f, context, size_t(S) * m.cfg.context_dim * 4, cudaMemcpyHostToDevice, s),
                 "context upload");
    MKB_TRY_CUDA(cast_f32_bf16(m.ctx_f, m.ctx_bf, size_t(S) * m.cfg.context_dim, s), "context cast");
    // Each transformer block's cross-attention keys and values of the context (sdxl.cpp:694-719).
    for (int t = 0; t < m.n_tblocks; ++t) {
        const int c = m.tb_c[t];
        const std::string name = [&] {
            int acc = 0;
            for (const auto& o : m.ops)
                if (o.kind == UnetImpl::Op::kAttn) {
                    if (t < acc + o.depth)
                        return o.name + ".b" + std::to_string(t - acc) + ".kv2.w";
                    acc += o.depth;
                }
            return std::string();
        }();
        const size_t off = size_t(slot) * c * S;
        GemmArgs a;
        a.M = S;
        a.N = 2 * c;
        a.K = m.cfg.context_dim;
        a.kh = m.kc[t] + off;
        a.vh = m.vc[t] + off;
        a.part0 = 1;
        a.D = c;
        a.head_dim = kHead;
        a.L = S;
        a.seg_rows = S;
        a.status = m.status;
        GemmOp op;
        const char* err = nullptr;
        if (!gemm_prepare(op, Epi::kHeads, m.ctx_bf, m.cfg.context_dim, m.W.M(name), m.cfg.context_dim, a,
                          (2 * c) % 128 == 0 ? 128 : 64, &err))
            return fail(MKB_ERR_INVALID, err ? err : "unet_begin: kv projection");
        MKB_TRY_CUDA(gemm_launch(op, s), "kv projection");
    }
    MKB_TRY_CUDA(cudaStreamSynchronize(s), "begin sync");
    m.ctx_rows[slot] = S;
    m.gh = gh;
    m.gw = gw;
    uint32_t bits = 0;
    MKB_TRY_CUDA(cudaMemcpy(&bits, m.status, 4, cudaMemcpyDeviceToHost), "status");
    if (bits)
        return fail(MKB_ERR_KERNEL, "unet_begin: kernel status " + std::to_string(bits));
    return MKB_OK;
}

mkb_status UnetImpl::run_step(int B, int slot0, const float* sigmas, cudaStream_t s)
{
    if (B < 1 || B > cfg.max_batch || slot0 < 0 || slot0 + B > cfg.slots)
        return fail(MKB_ERR_INVALID, "unet_step: batch out of range (sample i uses slot slot0 + i)");
    for (int i = 0; i < B; ++i)
        if (!ctx_rows[slot0 + i])
            return fail(MKB_ERR_STATE, "unet_step: step on a slot without begin");
    Plan* plan = nullptr;
    MKB_TRY(build(B, slot0, &plan));
    // Per sample: the timestep nearest sigma as a sinusoid, and the latents scaled by 1 / sqrt(sigma^2 + 1)
    // (sdxl.cpp:834-835).
    std::vector<float> ts(size_t(B) * C0);
    const size_t ntok = size_t(gh) * gw * 16;
    for (int i = 0; i < B; ++i)
        sinusoid_host(float(sdxl_schedule().timestep(sigmas[i])), C0, ts.data() + size_t(i) * C0);
    MKB_TRY_CUDA(cudaMemcpyAsync(tsin, ts.data(), ts.size() * 4, cudaMemcpyHostToDevice, s), "timestep upload");
    for (int i = 0; i < B; ++i) {
        const float sc = 1.0f / std::sqrt(sigmas[i] * sigmas[i] + 1.0f);
        MKB_TRY_CUDA(cfg_euler(tokens + i * ntok, tokens + i * ntok, nullptr, 0.0f, sc - 1.0f, ntok, s),
                     "latent scale");
    }
    return plan->run(s, probe, probe_user);
}

mkb_status mkb_unet_step_batch_dev(mkb_unet* u, int n, int slot0, const float* latents_dev, const float* sigmas,
                                   float* out_dev, void* stream)
{
    if (!u || !latents_dev || !sigmas || !out_dev)
        return fail(MKB_ERR_INVALID, "unet_step: null argument");
    UnetImpl& m = u->impl;
    if (n < 1 || n > m.cfg.max_batch)
        return fail(MKB_ERR_INVALID, "unet_step: batch out of range");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
    const size_t ntok = size_t(m.gh) * m.gw * 16;
    MKB_TRY_CUDA(cudaMemcpyAsync(m.tokens, latents_dev, size_t(n) * ntok * 4, cudaMemcpyDeviceToDevice, s), "latents");
    MKB_TRY(m.run_step(n, slot0, sigmas, s));
    MKB_TRY_CUDA(cudaMemcpyAsync(out_dev, m.eps_tok, size_t(n) * ntok * 4, cudaMemcpyDeviceToDevice, s), "eps copy");
    return MKB_OK;
}

mkb_status mkb_unet_step_batch(mkb_unet* u, int n, int slot0, const float* latents, const float* sigmas, float* out)
{
    if (!u || !latents || !sigmas || !out)
        return fail(MKB_ERR_INVALID, "unet_step: null argument");
    UnetImpl& m = u->impl;
    if (n < 1 || n > m.cfg.max_batch)
        return fail(MKB_ERR_INVALID, "unet_step: batch out of range");
    const size_t ntok = size_t(m.gh) * m.gw * 16;
    MKB_TRY_CUDA(cudaMemcpyAsync(m.tokens, latents, size_t(n) * ntok * 4, cudaMemcpyHostToDevice, m.stream),
                 "latents upload");
    MKB_TRY(m.run_step(n, slot0, sigmas, m.stream));
    MKB_TRY_CUDA(cudaMemcpyAsync(out, m.eps_tok, size_t(n) * ntok * 4, cudaMemcpyDeviceToHost, m.stream),
                 "eps download");
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "step sync");
    uint32_t bits = 0;
    MKB_TRY_CUDA(cudaMemcpy(&bits, m.status, 4, cudaMemcpyDeviceToHost), "status");
    if (bits) {
        cudaMemset(m.status, 0, 4);
        return fail(MKB_ERR_KERNEL, "unet_step: kernel status " + std::to_string(bits));
    }
    return MKB_OK;
}

mkb_status mkb_unet_step(mkb_unet* u, const float* latents, float sigma, float* out, int slot)
{
    return mkb_unet_step_batch(u, 1, slot, latents, &sigma, out);
}

mkb_status mkb_unet_step_cfg_dev(mkb_unet* u, float* latents_dev, float sigma, float sigma_next, float guidance,
                                 void* stream)
{
    if (!u || !latents_dev)
        return fail(MKB_ERR_INVALID, "unet_step_cfg: null argument");
    UnetImpl& m = u->impl;
    if (m.cfg.max_batch < 2 || m.cfg.slots < 2)
        return fail(MKB_ERR_INVALID, "unet_step_cfg: needs max_batch and slots >= 2");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
    const size_t ntok = size_t(m.gh) * m.gw * 16;
    // cond (slot 0) and uncond (slot 1) see the same latents, in one batched pass.
    MKB_TRY_CUDA(cudaMemcpyAsync(m.tokens, latents_dev, ntok * 4, cudaMemcpyDeviceToDevice, s), "latents");
    MKB_TRY_CUDA(cudaMemcpyAsync(m.tokens + ntok, latents_dev, ntok * 4, cudaMemcpyDeviceToDevice, s), "latents");
    const float sg[2] = {sigma, sigma};
    MKB_TRY(m.run_step(2, 0, sg, s));
    // Euler on the guided noise prediction (engine.cpp:476-480, 500-503).
    MKB_TRY_CUDA(cfg_euler(latents_dev, m.eps_tok, m.eps_tok + ntok, guidance, sigma_next - sigma, ntok, s),
                 "cfg euler");
    return MKB_OK;
}

mkb_status mkb_unet_set_probe(mkb_unet* u, mkb_probe_fn fn, void* user)
{
    if (!u)
        return fail(MKB_ERR_INVALID, "unet: null handle");
    u->impl.probe = fn;
    u->impl.probe_user = user;
    return MKB_OK;
}

double mkb_unet_step_flops(const mkb_unet* u, int n) { return u ? u->impl.flops(n) : 0.0; }

mkb_status mkb_sdxl_sigmas(uint32_t steps, float* out)
{
    if (!steps || !out)
        return fail(MKB_ERR_INVALID, "sdxl_sigmas: no steps");
    // Timesteps 999 -> 0 as a float linspace computes them (from both ends), log-sigma interpolated
    // (sdxl.cpp:653-670).
    const auto& sc = sdxl_schedule();
    const float start = 999.0f, end = 0.0f;
    const float stepv = steps > 1 ? (end - start) / float(steps - 1) : 0.0f;
    for (uint32_t i = 0; i < steps; ++i) {
        const float t = i < steps / 2 ? start + stepv * float(i) : end - stepv * float(steps - 1 - i);
        const float tc = std::min(std::max(t, 0.0f), 999.0f);
        const uint32_t lo = uint32_t(std::floor(tc)), hi = uint32_t(std::ceil(tc));
        const float wgt = tc - std::floor(tc);
        out[i] = std::exp((1.0f - wgt) * sc.log_sigma[lo] + wgt * sc.log_sigma[hi]);
    }
    out[steps] = 0.0f;
    return MKB_OK;
}

int mkb_sdxl_timestep(float sigma) { return sdxl_schedule().timestep(sigma); }

// ---------------------------------------------------------------------------------------------- VAE

mkb_status mkb_vae_create(const mkb_vae_config* cfg, mkb_vae** out)
{
    if (!cfg || !out)
        return fail(MKB_ERR_INVALID, "vae_create: null argument");
    auto* v = new (std::nothrow) mkb_vae;
    if (!v)
        return fail(MKB_ERR_ALLOC, "vae_create: host allocation");
    mkb_status s = v->impl.create(*cfg);
    if (s != MKB_OK) {
        delete v;
        return s;
    }
    *out = v;
    return MKB_OK;
}

void mkb_vae_destroy(mkb_vae* v)
{
    if (v) {
        cudaStreamSynchronize(v->impl.stream);
        delete v;
    }
}

mkb_status mkb_vae_init_random(mkb_vae* v, uint64_t seed, float std)
{
    if (!v)
        return fail(MKB_ERR_INVALID, "vae: null handle");
    return v->impl.W.init_random(seed, std, v->impl.stream);
}

int mkb_vae_weight_count(const mkb_vae* v) { return v ? int(v->impl.W.ws.size()) : 0; }

mkb_status mkb_vae_weight_info(const mkb_vae* v, int i, const char** name, long* dims, int* ndim)
{
    if (!v)
        return fail(MKB_ERR_INVALID, "vae: null handle");
    return v->impl.W.info(i, name, dims, ndim);
}

mkb_status mkb_vae_weight_read(mkb_vae* v, const char* name, float* host)
{
    if (!v || !name)
        return fail(MKB_ERR_INVALID, "vae: null argument");
    MKB_TRY_CUDA(cudaStreamSynchronize(v->impl.stream), "sync");
    return v->impl.W.read(name, host);
}

mkb_status mkb_vae_weight_write(mkb_vae* v, const char* name, const float* host)
{
    if (!v || !name)
        return fail(MKB_ERR_INVALID, "vae: null argument");
    MKB_TRY_CUDA(cudaStreamSynchronize(v->impl.stream), "sync");
    return v->impl.W.write(name, host);
}

mkb_status mkb_vae_decode_dev(mkb_vae* v, const float* latents_dev, int gh, int gw, float* rgba_dev, void* stream)
{
    if (!v || !latents_dev || !rgba_dev)
        return fail(MKB_ERR_INVALID, "vae_decode: null argument");
    VaeImpl& m = v->impl;
    if (gh < 1 || gw < 1 || gh > m.cfg.max_gh || gw > m.cfg.max_gw || (2 * gw) % 8)
        return fail(MKB_ERR_INVALID, "vae_decode: grid out of range (2 * gw a multiple of 8)");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
    Plan* plan = nullptr;
    MKB_TRY(m.build(gh, gw, &plan));
    MKB_TRY_CUDA(cudaMemcpyAsync(m.tokens, latents_dev, size_t(gh) * gw * 4 * m.z * 4, cudaMemcpyDeviceToDevice, s),
                 "latents");
    MKB_TRY(plan->run(s, m.probe, m.probe_user));
    MKB_TRY_CUDA(cudaMemcpyAsync(rgba_dev, m.rgba, size_t(gh) * gw * 256 * 4 * 4, cudaMemcpyDeviceToDevice, s),
                 "rgba copy");
    return MKB_OK;
}

mkb_status mkb_vae_decode(mkb_vae* v, const float* latents, int gh, int gw, float* rgba)
{
    if (!v || !latents || !rgba)
        return fail(MKB_ERR_INVALID, "vae_decode: null argument");
    VaeImpl& m = v->impl;
    if (gh < 1 || gw < 1 || gh > m.cfg.max_gh || gw > m.cfg.max_gw || (2 * gw) % 8)
        return fail(MKB_ERR_INVALID, "vae_decode: grid out of range (2 * gw a multiple of 8)");
    Plan* plan = nullptr;
    MKB_TRY(m.build(gh, gw, &plan));
    const size_t nt = size_t(gh) * gw * 4 * m.z, no = size_t(gh) * gw * 256 * 4;
    MKB_TRY_CUDA(cudaMemcpyAsync(m.tokens, latents, nt * 4, cudaMemcpyHostToDevice, m.stream), "latents upload");
    MKB_TRY(plan->run(m.stream, m.probe, m.probe_user));
    MKB_TRY_CUDA(cudaMemcpyAsync(rgba, m.rgba, no * 4, cudaMemcpyDeviceToHost, m.stream), "rgba download");
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "decode sync");
    uint32_t bits = 0;
    MKB_TRY_CUDA(cudaMemcpy(&bits, m.status, 4, cudaMemcpyDeviceToHost), "status");
    if (bits) {
        cudaMemset(m.status, 0, 4);
        return fail(MKB_ERR_KERNEL, "vae_decode: kernel status " + std::to_string(bits));
    }
    return MKB_OK;
}

mkb_status mkb_vae_set_probe(mkb_vae* v, mkb_probe_fn fn, void* user)
{
    if (!v)
        return fail(MKB_ERR_INVALID, "vae: null handle");
    v->impl.probe = fn;
    v->impl.probe_user = user;
    return MKB_OK;
}

double mkb_vae_decode_flops(const mkb_vae* v, int gh, int gw) { return v ? v->impl.flops(gh, gw) : 0.0; }

mkb_status mkb_vae_set_latent_stats(mkb_vae* v, const float* mean, const float* std, int n)
{
    if (!v || !mean || !std)
        return fail(MKB_ERR_INVALID, "vae_set_latent_stats: null argument");
    VaeImpl& m = v->impl;
    if (n != 4 * m.z)
        return fail(MKB_ERR_INVALID, "vae_set_latent_stats: need one mean and deviation per token value (4 x latent)");
    std::vector<float> aff(8 * m.z);
    for (int i = 0; i < n; ++i) {
        if (!(std[i] > 0) || !std::isfinite(mean[i]))
            return fail(MKB_ERR_INVALID, "vae_set_latent_stats: deviations must be positive, means finite");
        aff[i] = std[i];
        aff[4 * m.z + i] = mean[i];
    }
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "sync");
    MKB_TRY_CUDA(cudaMemcpy(m.lat_aff, aff.data(), aff.size() * 4, cudaMemcpyHostToDevice), "latent stats");
    return MKB_OK;
}

mkb_status mkb_clip_create(const mkb_clip_config* cfg, mkb_clip** out)
{
    if (!cfg || !out)
        return fail(MKB_ERR_INVALID, "clip_create: null argument");
    auto* c = new (std::nothrow) mkb_clip;
    if (!c)
        return fail(MKB_ERR_ALLOC, "clip_create: host allocation");
    mkb_status s = c->impl.create(*cfg);
    if (s != MKB_OK) {
        delete c;
        return s;
    }
    *out = c;
    return MKB_OK;
}

void mkb_clip_destroy(mkb_clip* c)
{
    if (c) {
        cudaStreamSynchronize(c->impl.stream);
        delete c;
    }
}

mkb_status mkb_clip_init_random(mkb_clip* c, uint64_t seed, float std)
{
    if (!c)
        return fail(MKB_ERR_INVALID, "clip: null handle");
    return c->impl.W.init_random(seed, std, c->impl.stream);
}

int mkb_clip_weight_count(const mkb_clip* c) { return c ? int(c->impl.W.ws.size()) : 0; }

mkb_status mkb_clip_weight_info(const mkb_clip* c, int i, const char** name, long* dims, int* ndim)
{
    if (!c)
        return fail(MKB_ERR_INVALID, "clip: null handle");
    return c->impl.W.info(i, name, dims, ndim);
}

mkb_status mkb_clip_weight_read(mkb_clip* c, const char* name, float* host)
{
    if (!c || !name)
        return fail(MKB_ERR_INVALID, "clip: null argument");
    MKB_TRY_CUDA(cudaStreamSynchronize(c->impl.stream), "sync");
    return c->impl.W.read(name, host);
}

mkb_status mkb_clip_weight_write(mkb_clip* c, const char* name, const float* host)
{
    if (!c || !name)
        return fail(MKB_ERR_INVALID, "clip: null argument");
    MKB_TRY_CUDA(cudaStreamSynchronize(c->impl.stream), "sync");
    return c->impl.W.write(name, host);
}

mkb_status mkb_clip_set_probe(mkb_clip* c, mkb_probe_fn fn, void* user)
{
    if (!c)
        return fail(MKB_ERR_INVALID, "clip: null handle");
    c->impl.probe = fn;
    c->impl.probe_user = user;
    return MKB_OK;
}

mkb_status mkb_clip_encode(mkb_clip* c, const int32_t* ids, int chunks, float* hidden, float* pooled)
{
    if (!c)
        return fail(MKB_ERR_INVALID, "clip: null handle");
    return c->impl.encode(ids, chunks, hidden, pooled);
}

mkb_status mkb_sdxl_prompt_embeddings(mkb_clip* l, mkb_clip* g, const int32_t* ids_l, const int32_t* ids_g,
                                      const float* weights, int chunks, float* context, float* pooled)
{
    if (!l || !g || !ids_l || !ids_g || !context || !pooled)
        return fail(MKB_ERR_INVALID, "prompt_embeddings: null argument");
    ClipImpl &L = l->impl, &G = g->impl;
    if (L.cfg.which != 0 || G.cfg.which != 1)
        return fail(MKB_ERR_INVALID, "prompt_embeddings: need the ViT-L handle (which 0) and the bigG one (which 1)");
    if (chunks < 1 || chunks > L.cfg.max_chunks || chunks > G.cfg.max_chunks)
        return fail(MKB_ERR_INVALID, "prompt_embeddings: chunk count out of range");
    const int EL = L.cfg.width, EG = G.cfg.width, T = kClipTokens;
    const size_t rows = size_t(chunks) * T;
    std::vector<float> zl(rows * EL), zg(rows * EG), pg(size_t(chunks) * kClipPooled);
    MKB_TRY(L.encode(ids_l, chunks, zl.data(), nullptr));
    MKB_TRY(G.encode(ids_g, chunks, zg.data(), pg.data()));
    bool weighted = false;
    for (size_t i = 0; weights && i < rows; ++i)
        weighted = weighted || weights[i] != 1.0f;
    std::vector<float> el, eg;
    if (weighted) {  // a weighted token's states move away from the empty prompt's by its weight (sdxl.cpp:618-631)
        std::vector<int32_t> e(T, kClipEnd);
        e[0] = kClipEnd - 1;
        el.resize(size_t(T) * EL);
        MKB_TRY(L.encode(e.data(), 1, el.data(), nullptr));
        std::fill(e.begin() + 2, e.end(), 0);
        eg.resize(size_t(T) * EG);
        std::vector<float> unused(kClipPooled);
        MKB_TRY(G.encode(e.data(), 1, eg.data(), unused.data()));
    }
    for (size_t r = 0; r < rows; ++r) {
        float* row = context + r * (EL + EG);
        const float w = weights ? weights[r] : 1.0f;
        const size_t t = r % T;
        for (int i = 0; i < EL; ++i) {
            const float z = zl[r * EL + i];
            row[i] = w != 1.0f ? (z - el[t * EL + i]) * w + el[t * EL + i] : z;
        }
        for (int i = 0; i < EG; ++i) {
            const float z = zg[r * EG + i];
            row[EL + i] = w != 1.0f ? (z - eg[t * EG + i]) * w + eg[t * EG + i] : z;
        }
    }
    std::copy(pg.begin(), pg.begin() + kClipPooled, pooled);  // the first chunk's pooled state
    return MKB_OK;
}

}  // extern "C"
