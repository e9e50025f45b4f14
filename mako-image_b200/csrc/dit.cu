// The denoiser handle behind include/mkb_image.h part 2: weights, step buffers and the per-step executor of the
// Qwen-Image-style MMDiT, in the reference's two block variants.
//
// The executor follows QwenImage::step (src/image/qwen_image.cpp:144-293) stage by stage, but every stage is one of
// this library's fused kernels: the time path runs as fp32-activation GEMVs, each projection is one tcgen05 GEMM
// whose epilogue applies bias / activation / gated residual / per-head RMSNorm + RoPE, LayerNorm-modulate is one
// warp-per-row pass, and attention is one flash kernel writing straight into the output projection's input.
#include "attention.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "launch.cuh"
#include "lora.cuh"
#include "nccl_dl.cuh"
#include "rowops.cuh"
#include "sm100.cuh"

#include <cmath>
#include <cstddef>
#include <cstring>
#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

namespace mkb {

namespace {

constexpr int kHeadDim = 128, kLatent = 64, kTimeDim = 256;
constexpr float kEps = 1e-6f;
constexpr size_t kSpFlagBytes = 512;  // the peer exchange's ready flags: one 64-bit word per rank, up to 64 ranks
constexpr size_t kHxFlagBytes = 1024; // the head exchange's: q|k|v stored [64], attention outputs stored [64]
constexpr int kSwigluBlock = 128;  // gate/up interleave of the SwiGLU GEMM (one 256-wide tile = 128 gate + 128 up)

uint64_t splitmix64_host(uint64_t x)
{
    uint64_t z = x + 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

struct Weight {
    std::string name;
    long rows = 0, cols = 0;  // cols == 0: vector
    size_t off = 0;           // element offset in its arena (bf16 matrices / fp32 vectors)
    bool swiglu = false;      // stored gate/up-interleaved
    bool norm = false;        // a norm scale (random init around 1)
    size_t count() const { return size_t(rows) * (cols ? cols : 1); }
};

// rope3 of the reference (qwen_image.cpp:31-45): 8 pairs on the frame axis, 28 each on height and width, theta 1e4.
void rope3(float* cs, long f, long hp, long wp)
{
    const int dims[3] = {16, 56, 56};
    const long pos[3] = {f, hp, wp};
    int i = 0;
    for (int a = 0; a < 3; ++a)
        for (int j = 0; j < dims[a] / 2; ++j, ++i) {
            const float inv = 1.0f / std::pow(10000.0f, float(2 * j) / float(dims[a]));
            const float ang = float(pos[a]) * inv;
            cs[2 * i] = std::cos(ang);
            cs[2 * i + 1] = std::sin(ang);
        }
}

// Sequence-parallel split of one sample's joint rows (text rows first, then image rows) over `world` ranks: rank r
// owns joint rows [r * Lg, (r + 1) * Lg). All text rows sit on rank 0 (S < Lg), so each rank runs one stream's
// weights on its image rows and rank 0 also the text stream's. Lg must be a multiple of 128 so that no attention key
// tile spans two ranks' shards.
struct SpRows {
    int text = 0;    // text rows on this rank (S on rank 0, else 0)
    int image = 0;   // image rows on this rank
    int image0 = 0;  // first image row (image-token index) on this rank
    int shard = 0;   // joint rows per rank, Lg
};

const char* sp_partition(int S, int N, int world, int rank, SpRows* out)
{
    if (world < 1 || rank < 0 || rank >= world || S < 1 || N < 1)
        return "sequence parallel: bad world, rank or token counts";
    const int L = S + N;
    if (L % world)
        return "sequence parallel: text + image tokens must divide evenly over the ranks";
    const int Lg = L / world;
    if (world > 1 && Lg % 128)
        return "sequence parallel: rows per rank must be a multiple of 128";
    if (S >= Lg && world > 1)
        return "sequence parallel: all text rows must fit on rank 0 with image rows to spare";
    out->shard = Lg;
    out->text = rank == 0 ? S : 0;
    out->image = Lg - out->text;
    out->image0 = rank * Lg - S + out->text;
    return nullptr;
}

}  // namespace

// The head-parallel exchange's per-rank destinations (a device table per plan, up to 64 ranks): where the QKV
// epilogue stores each rank's heads, where the attention stores each rank's rows, and (peer-memory mode) the flags
// this rank raises in every peer's region.
struct HxTables {
    __nv_bfloat16* group_dst[64];
    AttnOutShard out[64];
    unsigned long long* sig_qkv[64];
    unsigned long long* sig_att[64];
};

struct DitImpl {
    mkb_dit_config cfg{};
    int D = 0, H = 0, F = 0, NB = 0, TD = 0;
    int Bmax = 0, Smax = 0, Nmax = 0, Lmax = 0;
    cudaStream_t stream = nullptr;
    uint32_t* status = nullptr;
    // qwen1: block i's modulation GEMV (i >= 1) runs on a side stream beside the blocks before it (its blocks use no
    // shared memory, so they fit on SMs beside the GEMMs' CTAs), joined before block i; block 0's on the step's stream.
    cudaStream_t mod_side = nullptr;
    cudaEvent_t mod_fork = nullptr;
    std::vector<cudaEvent_t> mod_ready;

    std::vector<Weight> weights;
    std::map<std::string, int> windex;
    __nv_bfloat16* wmat = nullptr;
    float* wvec = nullptr;
    size_t wmat_n = 0, wvec_n = 0;

    // step buffers
    float *x_txt = nullptr, *x_img = nullptr, *vel = nullptr, *lat = nullptr;
    __nv_bfloat16 *xn = nullptr, *qh = nullptr, *kh = nullptr, *vh = nullptr, *attn = nullptr, *hid = nullptr;
    __nv_bfloat16 *lat_bf = nullptr, *txt_bf = nullptr, *txt_mid = nullptr;
    float *tp = nullptr, *h1 = nullptr, *temb = nullptr, *st = nullptr, *mod = nullptr, *omod = nullptr;
    float *sig = nullptr, *rope = nullptr;
    float* cfg_lat = nullptr;  // device copy of one image's latents for the host-buffer guided step

    struct Slot {
        bool begun = false;
        int S = 0, steps = 0;
        float* prompt = nullptr;                    // device [Smax][TD]
        std::vector<__nv_bfloat16*> kc, vc;         // ref21 text K/V per block, [H][S][128]
    };
    std::vector<Slot> slots;
    int gh = 0, gw = 0;
    long rope_key[3] = {-1, -1, -1};

    mkb_probe_fn probe = nullptr;
    void* probe_user = nullptr;

    // Prepared launches per geometry (batch, text rows, image rows, first step of ref21).
    struct Plan {
        std::vector<GemmOp> ops;  // indexed by the builder
        AttnOp att;
        AttnOp att_odd;  // odd blocks' attention under the peer exchange (the second K/V buffer)
        std::vector<GemmOp> per_sample;  // ref21 txt_in2 / img_in per sample
        HxTables* tab = nullptr;  // device copy: the head exchange's destinations for this geometry
        ~Plan()
        {
            if (tab)
                cudaFree(tab);
        }
    };
    std::map<std::tuple<int, int, int, int>, std::unique_ptr<Plan>> plans;

    // The step body captured as a CUDA graph per (batch, prompt rows, image rows, first step, slots): the first call
    // of a key runs eagerly (it sets kernel attributes and plans), the second captures, later ones replay.
    struct Graph {
        int seen = 0;
        cudaGraphExec_t exec = nullptr;
        unsigned long long launches = 0;
    };
    std::map<std::vector<int>, Graph> graphs;
    bool use_graphs = true;

    // Sequence parallelism (qwen1): this rank's share of every sample's joint rows; per block the ranks all-gather
    // their K and V shards (the QKV epilogue writes them straight into this rank's slot of kv_all).
    int sp_world = 1, sp_rank = 0;
    ncclComm_t sp_comm = nullptr;
    int sp_lg_max = 0;
    __nv_bfloat16* kv_all = nullptr;  // [world][2 (K, V)][B][H][Lg][128] for the step's B and Lg
    float* vel_x = nullptr;           // [world][B][Lg][64]: velocity exchange
    float* vel_full = nullptr;        // [Bmax][Nmax][64]: all image rows' velocities after the exchange
    // Peer-memory exchange of the K/V shards (replaces the per-block all-gather): the QKV epilogue writes this rank's
    // shard into its slot of this GPU's exchange region; one copy stream per peer pushes the slot into that peer's
    // region (the copies run side by side on the copy engines: one at a time would move ~1/7 of the link bandwidth at
    // eight ranks) and then raises this rank's ready flag there; the attention waits on the flags. Blocks alternate
    // between two K/V buffers, so no push lands in a buffer a peer still reads: this rank pushes block i + 2 after
    // its attention of block i + 1, which waited for the peer's block-(i + 1) shard, which the peer pushes only after
    // its own attention of block i. The copies run on copy engines, not SMs, so they overlap the attention.
    bool sp_p2p = false;
    uint8_t* sp_region = nullptr;          // [ready flags, kSpFlagBytes][K/V, even blocks][K/V, odd blocks]
    size_t sp_kv_bytes = 0;                // one K/V buffer: [world][2][Bmax][H][sp_lg_max][128] bf16
    std::vector<uint8_t*> sp_peer;         // every rank's region as mapped in this process (own region at sp_rank)
    unsigned long long* sp_seq = nullptr;  // [0] steps run, [1 + i] the ready value of block i in the current step
    std::vector<cudaStream_t> sp_side;     // the pushes, one stream per peer
    cudaEvent_t sp_fork = nullptr;
    std::vector<cudaEvent_t> sp_done[2];   // per block parity, per copy stream: the pushes done
    __nv_bfloat16* kv_buf(int parity) const
    {
        return reinterpret_cast<__nv_bfloat16*>(sp_region + kSpFlagBytes + parity * sp_kv_bytes);
    }
    mkb_status sp_set_peer(bool on);
    void sp_release_peer();
    mkb_status sp_push(int B, int Lg, int block, cudaStream_t s);
    // Head-parallel exchange (replaces the K/V all-gather; H divisible by the ranks): after each block's QKV
    // projection an all-to-all gives every rank all joint rows of its H / world heads (the QKV epilogue writes the
    // rows of rank g's heads into span g of the send buffer, its own heads straight into the receive buffer), the
    // attention runs over whole sequences for those heads, and a second all-to-all returns each rank's rows of
    // every head. Per block a rank receives 4 (world - 1) / world^2 of one step-wide activation instead of the
    // all-gather's 2 (world - 1) / world, and every row sees its keys in the one-GPU order.
    // Mode 1 moves the spans with NCCL (send and receive buffers in sp_hx, outputs gathered into the O projection's
    // rows by a copy kernel); mode 2 stores them straight into the peers' memory from the QKV and attention
    // epilogues (every rank's IPC region holds [flags][q|k|v receive][the O projection's input rows], the
    // attention waits for each peer's q|k|v flag before its first tile of that peer's rows, and the O projection
    // waits for every peer's attention-done flag).
    int sp_heads = 0;
    __nv_bfloat16* sp_hx = nullptr;  // mode 1: [q|k|v send][q|k|v receive][output send][output receive]
    size_t sp_hx_qkv = 0;            // elements of one q|k|v buffer: [world][3][B][H / world][Lg][128]
    size_t sp_hx_o = 0;              // elements of one output buffer: [world][B][Lg][H / world * 128]
    __nv_bfloat16* hx_region_qkv(int g) const  // mode 2: rank g's q|k|v receive buffer, as mapped here
    {
        return reinterpret_cast<__nv_bfloat16*>(sp_peer[g] + kHxFlagBytes);
    }
    __nv_bfloat16* hx_region_rows(int g) const  // mode 2: rank g's O projection input rows
    {
        return hx_region_qkv(g) + sp_hx_qkv;
    }
    bool sp_open_region(size_t bytes, bool ok, std::string* why);
    mkb_status sp_set_heads(int mode);
    mkb_status sp_all_to_all(const __nv_bfloat16* send, __nv_bfloat16* recv, size_t count, cudaStream_t s);
    bool sp_agree(bool ok);
    SpRows rows_of(int S, int N) const
    {
        SpRows r;
        if (sp_world > 1)
            sp_partition(S, N, sp_world, sp_rank, &r);
        else
            r = SpRows{S, N, 0, S + N};
        return r;
    }
    mkb_status set_sp(const void* id, int rank, int world);
    mkb_status sp_gather_velocity(int B, int S, float* out, cudaMemcpyKind kind, cudaStream_t s);
    mkb_status stage_latents(int n_src, int copies, int S, const float* src, cudaMemcpyKind kind, cudaStream_t s);

    ~DitImpl();
    mkb_status create(const mkb_dit_config& c);
    void add_weight(const std::string& name, long rows, long cols, bool norm = false, bool swiglu = false);
    const Weight* find(const std::string& n) const
    {
        auto it = windex.find(n);
        return it == windex.end() ? nullptr : &weights[it->second];
    }
    const __nv_bfloat16* M(const std::string& n) const { return wmat + find(n)->off; }
    const float* V(const std::string& n) const
    {
        const Weight* w = find(n);
        return w ? wvec + w->off : nullptr;
    }
    mkb_status build_plan(int B, int S, int N, int first, Plan** out);
    mkb_status run(int B, const int* slot_ids, const float* sigmas, cudaStream_t s, bool* first_out);
    mkb_status body(int B, const int* slot_ids, int S, int N, int first, Plan* plan, cudaStream_t s);
    mkb_status upload_rope(int S, cudaStream_t s);
    mkb_status emit(const char* name, int layer, const float* dev, long count, cudaStream_t s);
    mkb_status check_status();
};

DitImpl::~DitImpl()
{
    void* bufs[] = {wmat, wvec, x_txt, x_img, vel, lat, xn, qh, kh, vh, attn, hid, lat_bf, txt_bf, txt_mid,
                    tp, h1, temb, st, mod, omod, sig, rope, cfg_lat, kv_all, vel_x, vel_full, sp_hx};
    if (stream)
        cudaStreamSynchronize(stream);
    for (void* p : bufs)
        if (p)
            cudaFree(p);
    for (auto& s : slots) {
        if (s.prompt)
            cudaFree(s.prompt);
        for (auto* p : s.kc)
            cudaFree(p);
        for (auto* p : s.vc)
            cudaFree(p);
    }
    // Graphs may hold the communicator's collectives: release them before the communicator.
    for (auto& g : graphs)
        if (g.second.exec)
            cudaGraphExecDestroy(g.second.exec);
    sp_release_peer();
    if (sp_comm) {
        if (const NcclApi* api = nccl_api(nullptr))
            api->CommDestroy(sp_comm);
    }
    if (mod_side)
        cudaStreamSynchronize(mod_side);
    for (cudaEvent_t e : mod_ready)
        if (e)
            cudaEventDestroy(e);
    if (mod_fork)
        cudaEventDestroy(mod_fork);
    if (mod_side)
        cudaStreamDestroy(mod_side);
    if (stream)
        cudaStreamDestroy(stream);
}

mkb_status DitImpl::set_sp(const void* id, int rank, int world)
{
    if (cfg.variant != MKB_VARIANT_QWEN1)
        return fail(MKB_ERR_INVALID, "sequence parallel: qwen1 variant only");
    if (world < 1 || world > 64 || rank < 0 || rank >= world)
        return fail(MKB_ERR_INVALID, "sequence parallel: need 1 <= world <= 64 and 0 <= rank < world");
    if (sp_comm || sp_world > 1)
        return fail(MKB_ERR_STATE, "sequence parallel: already set on this handle");
    if (world == 1)
        return MKB_OK;
    if (!id)
        return fail(MKB_ERR_INVALID, "sequence parallel: null NCCL id");
    std::string err;
    const NcclApi* api = nccl_api(&err);
    if (!api)
        return fail(MKB_ERR_CUDA, "sequence parallel: " + err);
    sp_lg_max = ((Lmax + world - 1) / world + 127) / 128 * 128;
    // On any failure below the handle stays as it was: the exchange buffers are released again.
    auto release = [&] {
        for (void** p : {reinterpret_cast<void**>(&kv_all), reinterpret_cast<void**>(&vel_x),
                         reinterpret_cast<void**>(&vel_full)}) {
            if (*p)
                cudaFree(*p);
            *p = nullptr;
        }
    };
    const size_t B = Bmax;
    const size_t kv = size_t(world) * 2 * B * H * sp_lg_max * kHeadDim * 2;
    const size_t vx = size_t(world) * B * sp_lg_max * kLatent * 4, vf = B * size_t(Nmax) * kLatent * 4;
    for (auto [p, bytes, what] : {std::tuple<void**, size_t, const char*>{reinterpret_cast<void**>(&kv_all), kv, "kv"},
                                  {reinterpret_cast<void**>(&vel_x), vx, "velocity exchange"},
                                  {reinterpret_cast<void**>(&vel_full), vf, "velocities"}}) {
        cudaError_t e = cudaMalloc(p, bytes);
        if (e != cudaSuccess) {
            cudaGetLastError();  // not sticky: keep it out of later launch checks
            release();
            return fail(MKB_ERR_ALLOC, std::string("sequence parallel: allocating ") + what + ": " +
                                           cudaGetErrorString(e));
        }
    }
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    ncclComm_t comm = nullptr;
    const ncclResult_t r = api->CommInitRank(&comm, world, uid, rank);
    if (r != ncclSuccess) {
        release();
        return fail(MKB_ERR_CUDA, std::string("sequence parallel: ncclCommInitRank: ") + api->GetErrorString(r));
    }
    sp_comm = comm;
    sp_world = world;
    sp_rank = rank;
    // Plans and graphs were built for the unsplit geometry.
    for (auto& g : graphs)
        if (g.second.exec)
            cudaGraphExecDestroy(g.second.exec);
    graphs.clear();
    plans.clear();
    return MKB_OK;
}

void DitImpl::sp_release_peer()
{
    for (cudaStream_t x : sp_side)
        if (x)
            cudaStreamSynchronize(x);
    for (int g = 0; g < int(sp_peer.size()); ++g)
        if (sp_peer[g] && g != sp_rank)
            cudaIpcCloseMemHandle(sp_peer[g]);
    sp_peer.clear();
    for (auto& v : sp_done) {
        for (cudaEvent_t e : v)
            if (e)
                cudaEventDestroy(e);
        v.clear();
    }
    if (sp_fork)
        cudaEventDestroy(sp_fork);
    sp_fork = nullptr;
    for (cudaStream_t x : sp_side)
        if (x)
            cudaStreamDestroy(x);
    sp_side.clear();
    if (sp_region)
        cudaFree(sp_region);
    if (sp_seq)
        cudaFree(sp_seq);
    sp_region = nullptr;
    sp_seq = nullptr;
    sp_p2p = false;
    cudaGetLastError();  // a failed set-up step is reported by the caller, not by later launches
}

// Allocates this rank's exchange region (`bytes`, zeroed), exports it over CUDA IPC, gathers every rank's handle
// (an NCCL all-gather through the idle velocity buffer) and maps the peers' regions into sp_peer (own region at
// sp_rank). `ok` carries this rank's earlier set-up into the first agreement; a second one follows the mapping.
// Every rank returns the same answer; on false *why holds this rank's reason (empty: another rank failed), and the
// caller releases what was made.
bool DitImpl::sp_open_region(size_t bytes, bool ok, std::string* why)
{
    const NcclApi* api = nccl_api(nullptr);
    struct Entry {
        cudaIpcMemHandle_t h;
        int ok;
        int pad[15];
    };
    auto step = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && why->empty())
            *why = std::string(what) + ": " + cudaGetErrorString(e);
        return e == cudaSuccess;
    };
    Entry mine{};
    ok = ok && step(cudaMalloc(&sp_region, bytes), "allocating the exchange region") &&
         step(cudaMemsetAsync(sp_region, 0, bytes, stream), "clearing it") &&
         step(cudaIpcGetMemHandle(&mine.h, sp_region), "cudaIpcGetMemHandle");
    mine.ok = ok;
    std::vector<Entry> all(sp_world);
    auto gather = [&](const Entry& e) -> bool {
        Entry* buf = reinterpret_cast<Entry*>(vel_x);  // the velocity exchange buffer, idle between steps
        if (cudaMemcpyAsync(buf + sp_rank, &e, sizeof(Entry), cudaMemcpyHostToDevice, stream) != cudaSuccess)
            return false;
        if (api->AllGather(buf + sp_rank, buf, sizeof(Entry), ncclUint8, sp_comm, stream) != ncclSuccess)
            return false;
        return cudaMemcpyAsync(all.data(), buf, sizeof(Entry) * sp_world, cudaMemcpyDeviceToHost, stream) ==
                   cudaSuccess &&
               cudaStreamSynchronize(stream) == cudaSuccess;
    };
    auto all_ok = [&] {
        for (const Entry& e : all)
            if (!e.ok)
                return false;
        return true;
    };
    if (!gather(mine) || !all_ok())
        return false;
    sp_peer.assign(sp_world, nullptr);
    sp_peer[sp_rank] = sp_region;
    const std::vector<Entry> handles = all;
    bool opened = true;
    for (int g = 0; g < sp_world && opened; ++g) {
        if (g == sp_rank)
            continue;
        void* p = nullptr;
        opened = step(cudaIpcOpenMemHandle(&p, handles[g].h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
        sp_peer[g] = static_cast<uint8_t*>(p);
    }
    Entry e2{};
    e2.ok = opened;
    return gather(e2) && all_ok();
}

// Switches the K/V exchange between the NCCL all-gather and peer memory. Collective over the group: every rank
// calls it with the same `on`. Each rank exports its exchange region over CUDA IPC, the handles go round by an
// all-gather, and every rank maps the others'; a second all-gather makes every rank fail together if any could not.
mkb_status DitImpl::sp_set_peer(bool on)
{
    if (sp_world < 2 || !sp_comm)
        return fail(MKB_ERR_STATE, "peer exchange: set sequence parallelism first");
    if (on == sp_p2p)
        return MKB_OK;
    if (on && sp_heads)
        MKB_TRY(sp_set_heads(0));
    MKB_TRY_CUDA(cudaStreamSynchronize(stream), "peer exchange: sync");
    for (auto& g : graphs)  // plans and graphs hold the K/V buffers of the other mode
        if (g.second.exec)
            cudaGraphExecDestroy(g.second.exec);
    graphs.clear();
    plans.clear();
    if (!on) {
        sp_release_peer();
        return MKB_OK;
    }
    sp_kv_bytes = (size_t(sp_world) * 2 * Bmax * H * sp_lg_max * kHeadDim * 2 + 255) / 256 * 256;
    std::string why;
    auto step = [&](cudaError_t e, const char* what) {
        if (e != cudaSuccess && why.empty())
            why = std::string(what) + ": " + cudaGetErrorString(e);
        return e == cudaSuccess;
    };
    bool ok = step(cudaMalloc(&sp_seq, (1 + size_t(NB)) * 8), "allocating the block counters") &&
              step(cudaMemsetAsync(sp_seq, 0, (1 + size_t(NB)) * 8, stream), "clearing them") &&
              step(cudaEventCreateWithFlags(&sp_fork, cudaEventDisableTiming), "events");
    sp_side.assign(sp_world - 1, nullptr);
    for (auto& v : sp_done)
        v.assign(sp_world - 1, nullptr);
    for (int k = 0; k < sp_world - 1; ++k) {
        ok = ok && step(cudaStreamCreateWithFlags(&sp_side[k], cudaStreamNonBlocking), "copy streams");
        for (auto& v : sp_done)
            ok = ok && step(cudaEventCreateWithFlags(&v[k], cudaEventDisableTiming), "events");
    }
    if (!sp_open_region(kSpFlagBytes + 2 * sp_kv_bytes, ok, &why)) {
        sp_release_peer();
        return fail(MKB_ERR_CUDA, "peer exchange: " + (why.empty() ? std::string("another rank failed") : why));
    }
    sp_p2p = true;
    return MKB_OK;
}

// The pushes of block `block`'s K/V shard (this rank's slot of its buffer) into every peer's region, each followed by
// the 8-byte copy of the block's ready value into the peer's flag of this rank, on the copy stream (forked from s
// after the QKV projection that wrote the shard).
mkb_status DitImpl::sp_push(int B, int Lg, int block, cudaStream_t s)
{
    const size_t shard = size_t(2) * B * H * Lg * kHeadDim * 2;
    const size_t off = kSpFlagBytes + size_t(block & 1) * sp_kv_bytes + size_t(sp_rank) * shard;
    MKB_TRY_CUDA(cudaEventRecord(sp_fork, s), "push fork");
    for (int k = 1; k < sp_world; ++k) {
        const int q = (sp_rank - k + sp_world) % sp_world;
        cudaStream_t x = sp_side[k - 1];
        MKB_TRY_CUDA(cudaStreamWaitEvent(x, sp_fork, 0), "push fork");
        MKB_TRY_CUDA(cudaMemcpyAsync(sp_peer[q] + off, sp_region + off, shard, cudaMemcpyDeviceToDevice, x),
                     "K/V push");
        MKB_TRY_CUDA(cudaMemcpyAsync(sp_peer[q] + size_t(sp_rank) * 8, sp_seq + 1 + block, 8,
                                     cudaMemcpyDeviceToDevice, x),
                     "ready flag");
        MKB_TRY_CUDA(cudaEventRecord(sp_done[block & 1][k - 1], x), "push done");
    }
    return MKB_OK;
}

// True on every rank when every rank passes ok: a one-word all-gather through the velocity exchange buffer.
bool DitImpl::sp_agree(bool ok)
{
    const NcclApi* api = nccl_api(nullptr);
    int* buf = reinterpret_cast<int*>(vel_x);  // idle between steps
    std::vector<int> all(sp_world, 0);
    const int mine = ok ? 1 : 0;
    if (cudaMemcpyAsync(buf + sp_rank, &mine, sizeof(int), cudaMemcpyHostToDevice, stream) != cudaSuccess ||
        api->AllGather(buf + sp_rank, buf, 1, ncclInt32, sp_comm, stream) != ncclSuccess ||
        cudaMemcpyAsync(all.data(), buf, sizeof(int) * sp_world, cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
        cudaStreamSynchronize(stream) != cudaSuccess)
        return false;
    for (int v : all)
        if (!v)
            return false;
    return true;
}

// Switches to the head-parallel exchange (mode 1: NCCL all-to-all, 2: stores into the peers' memory) or back to the
// K/V all-gather (0). Collective: every rank with the same mode.
mkb_status DitImpl::sp_set_heads(int mode)
{
    if (sp_world < 2 || !sp_comm)
        return fail(MKB_ERR_STATE, "head exchange: set sequence parallelism first");
    if (mode < 0 || mode > 2)
        return fail(MKB_ERR_INVALID, "head exchange: mode must be 0, 1 or 2");
    if (mode == sp_heads)
        return MKB_OK;
    if (mode && H % sp_world)
        return fail(MKB_ERR_INVALID, "head exchange: the heads must divide evenly over the ranks");
    if (sp_p2p)
        MKB_TRY(sp_set_peer(false));
    MKB_TRY_CUDA(cudaStreamSynchronize(stream), "head exchange: sync");
    for (auto& g : graphs)  // plans and graphs hold the buffers of the other mode
        if (g.second.exec)
            cudaGraphExecDestroy(g.second.exec);
    graphs.clear();
    plans.clear();
    if (sp_hx)
        cudaFree(sp_hx);
    sp_hx = nullptr;
    sp_release_peer();
    sp_heads = 0;
    if (!mode)
        return MKB_OK;
    sp_hx_qkv = size_t(3) * Bmax * H * sp_lg_max * kHeadDim;
    sp_hx_o = size_t(Bmax) * sp_lg_max * H * kHeadDim;
    if (mode == 1) {
        const cudaError_t e = cudaMalloc(&sp_hx, (2 * sp_hx_qkv + 2 * sp_hx_o) * sizeof(__nv_bfloat16));
        if (e != cudaSuccess) {
            cudaGetLastError();
            sp_hx = nullptr;
        }
        if (!sp_agree(e == cudaSuccess)) {
            if (sp_hx)
                cudaFree(sp_hx);
            sp_hx = nullptr;
            return fail(e == cudaSuccess ? MKB_ERR_CUDA : MKB_ERR_ALLOC,
                        e == cudaSuccess ? std::string("head exchange: another rank failed")
                                         : std::string("head exchange: allocating: ") + cudaGetErrorString(e));
        }
    } else {
        std::string why;
        const bool ok = cudaMalloc(&sp_seq, (1 + size_t(NB)) * 8) == cudaSuccess &&
                        cudaMemsetAsync(sp_seq, 0, (1 + size_t(NB)) * 8, stream) == cudaSuccess;
        if (!ok)
            why = "allocating the block counters";
        if (!sp_open_region(kHxFlagBytes + (sp_hx_qkv + sp_hx_o) * sizeof(__nv_bfloat16), ok, &why)) {
            cudaGetLastError();
            sp_release_peer();
            return fail(MKB_ERR_CUDA, "head exchange: " + (why.empty() ? std::string("another rank failed") : why));
        }
    }
    sp_heads = mode;
    return MKB_OK;
}

// All-to-all of `count` elements per rank pair: span g of `send` to rank g, rank g's span into span g of `recv`.
// This rank's own span is written in place by the producer and not copied.
mkb_status DitImpl::sp_all_to_all(const __nv_bfloat16* send, __nv_bfloat16* recv, size_t count, cudaStream_t s)
{
    const NcclApi* api = nccl_api(nullptr);
    ncclResult_t r = api->GroupStart();
    for (int k = 1; k < sp_world && r == ncclSuccess; ++k) {
        const int to = (sp_rank + k) % sp_world, from = (sp_rank - k + sp_world) % sp_world;
        r = api->Send(send + size_t(to) * count, count, ncclBfloat16, to, sp_comm, s);
        if (r == ncclSuccess)
            r = api->Recv(recv + size_t(from) * count, count, ncclBfloat16, from, sp_comm, s);
    }
    const ncclResult_t r2 = api->GroupEnd();
    if (r == ncclSuccess)
        r = r2;
    if (r != ncclSuccess)
        return fail(MKB_ERR_CUDA, std::string("dit: head exchange all-to-all: ") + api->GetErrorString(r));
    return MKB_OK;
}

void DitImpl::add_weight(const std::string& name, long rows, long cols, bool norm, bool swiglu)
{
    Weight w;
    w.name = name;
    w.rows = rows;
    w.cols = cols;
    w.norm = norm;
    w.swiglu = swiglu;
    if (cols) {
        w.off = wmat_n;
        wmat_n += size_t(rows) * cols;
    } else {
        w.off = wvec_n;
        wvec_n += size_t(rows);
        wvec_n = (wvec_n + 3) & ~size_t(3);  // keep every vector 16-byte aligned
    }
    windex[name] = int(weights.size());
    weights.push_back(w);
}

mkb_status DitImpl::create(const mkb_dit_config& c)
{
    cfg = c;
    D = c.hidden;
    H = c.heads;
    F = c.ffn;
    NB = c.blocks;
    TD = c.text_dim;
    Bmax = c.max_batch;
    Smax = c.max_text_tokens;
    Nmax = c.max_image_tokens;
    Lmax = Smax + Nmax;
    if (c.variant != MKB_VARIANT_QWEN1 && c.variant != MKB_VARIANT_REF21)
        return fail(MKB_ERR_INVALID, "dit: unknown variant");
    if (H <= 0 || D != H * kHeadDim || D % 256 || F <= 0 || F % 256 || NB <= 0 || TD <= 0 || TD % 128 ||
        TD > 4096 || D > 4096)
        return fail(MKB_ERR_INVALID, "dit: need hidden = heads * 128 (a multiple of 256, <= 4096), ffn a multiple "
                                     "of 256, text_dim a multiple of 128 (<= 4096), blocks > 0");
    if (Bmax < 1 || Bmax > 8 || Smax < 1 || Nmax < 1 || c.slots < 1)
        return fail(MKB_ERR_INVALID, "dit: need 1 <= max_batch <= 8, max tokens >= 1, slots >= 1");
    const bool q1 = c.variant == MKB_VARIANT_QWEN1;

    // Weight table. The per-block modulation matrices come first so all of them form one stacked GEMV operand.
    if (q1) {
        for (int i = 0; i < NB; ++i)
            for (const char* s : {"img", "txt"}) {
                const std::string p = "blk" + std::to_string(i) + "." + s + ".";
                add_weight(p + "mod.w", 6L * D, D);
                add_weight(p + "mod.b", 6L * D, 0);
            }
        add_weight("time.lin1.w", D, kTimeDim);
        add_weight("time.lin1.b", D, 0);
        add_weight("time.lin2.w", D, D);
        add_weight("time.lin2.b", D, 0);
        add_weight("img_in.w", D, kLatent);
        add_weight("img_in.b", D, 0);
        add_weight("txt_norm.w", TD, 0, true);
        add_weight("txt_in.w", D, TD);
        add_weight("txt_in.b", D, 0);
        add_weight("norm_out.w", 2L * D, D);
        add_weight("norm_out.b", 2L * D, 0);
        add_weight("proj_out.w", kLatent, D);
        add_weight("proj_out.b", kLatent, 0);
        for (int i = 0; i < NB; ++i)
            for (const char* s : {"img", "txt"}) {
                const std::string p = "blk" + std::to_string(i) + "." + s + ".";
                add_weight(p + "qkv.w", 3L * D, D);
                add_weight(p + "qkv.b", 3L * D, 0);
                add_weight(p + "norm_q", kHeadDim, 0, true);
                add_weight(p + "norm_k", kHeadDim, 0, true);
                add_weight(p + "o.w", D, D);
                add_weight(p + "o.b", D, 0);
                add_weight(p + "ff1.w", F, D);
                add_weight(p + "ff1.b", F, 0);
                add_weight(p + "ff2.w", D, F);
                add_weight(p + "ff2.b", D, 0);
            }
    } else {
        add_weight("time.lin1.w", D, kTimeDim);
        add_weight("time.lin2.w", D, D);
        add_weight("mod.w", 4L * D, D);
        add_weight("img_in.w", D, kLatent);
        add_weight("txt_norm.w", TD, 0, true);
        add_weight("txt_in1.w", D, TD);
        add_weight("txt_in2.w", D, D);
        add_weight("norm_out.w", D, D);
        add_weight("proj_out.w", kLatent, D);
        for (int i = 0; i < NB; ++i) {
            const std::string p = "blk" + std::to_string(i) + ".";
            add_weight(p + "qkv.w", 3L * D, D);
            add_weight(p + "norm_q", kHeadDim, 0, true);
            add_weight(p + "norm_k", kHeadDim, 0, true);
            add_weight(p + "o.w", D, D);
            add_weight(p + "gate_up.w", 2L * F, D, false, true);
            add_weight(p + "down.w", D, F);
        }
    }

    MKB_TRY_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    if (q1) {
        MKB_TRY_CUDA(cudaStreamCreateWithFlags(&mod_side, cudaStreamNonBlocking), "modulation stream");
        MKB_TRY_CUDA(cudaEventCreateWithFlags(&mod_fork, cudaEventDisableTiming), "modulation events");
        mod_ready.assign(NB, nullptr);
        for (auto& e : mod_ready)
            MKB_TRY_CUDA(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "modulation events");
    }
    status = device_status_word();
    if (!status)
        return fail(MKB_ERR_CUDA, "status word");
    auto alloc = [&](void** p, size_t bytes, const char* what) -> mkb_status {
        cudaError_t e = cudaMalloc(p, bytes ? bytes : 16);
        if (e != cudaSuccess) {
            cudaGetLastError();  // not sticky: keep it out of later launch checks
            return fail(MKB_ERR_ALLOC, std::string("dit: allocating ") + what + ": " + cudaGetErrorString(e));
        }
        return MKB_OK;
    };
#define MKB_ALLOC(ptr, bytes)                                                                                          \
    do {                                                                                                               \
        mkb_status s_ = alloc(reinterpret_cast<void**>(&ptr), (bytes), #ptr);                                          \
        if (s_ != MKB_OK)                                                                                              \
            return s_;                                                                                                 \
    } while (0)
    MKB_ALLOC(wmat, wmat_n * 2);
    MKB_ALLOC(wvec, wvec_n * 4);
    MKB_TRY_CUDA(cudaMemset(wmat, 0, wmat_n * 2), "zero weights");
    MKB_TRY_CUDA(cudaMemset(wvec, 0, wvec_n * 4), "zero weights");
    const size_t B = Bmax, L = Lmax;
    MKB_ALLOC(x_txt, B * Smax * D * 4);
    MKB_ALLOC(x_img, B * L * D * 4);
    MKB_ALLOC(xn, B * L * D * 2);
    MKB_ALLOC(qh, B * H * L * kHeadDim * 2);
    MKB_ALLOC(kh, B * H * L * kHeadDim * 2);
    MKB_ALLOC(vh, B * H * L * kHeadDim * 2);
    MKB_ALLOC(attn, B * L * D * 2);
    MKB_ALLOC(hid, B * L * F * 2);
    MKB_ALLOC(vel, B * L * kLatent * 4);
    MKB_ALLOC(lat, B * Nmax * kLatent * 4);
    MKB_ALLOC(lat_bf, B * Nmax * kLatent * 2);
    MKB_ALLOC(txt_bf, B * Smax * TD * 2);
    MKB_ALLOC(txt_mid, B * Smax * D * 2);
    MKB_ALLOC(tp, 2 * B * kTimeDim * 4);
    MKB_ALLOC(h1, 2 * B * D * 4);
    MKB_ALLOC(temb, 2 * B * D * 4);
    MKB_ALLOC(st, 2 * B * D * 4);
    MKB_ALLOC(mod, q1 ? B * NB * 12 * D * 4 : 2 * B * 4 * D * 4);
    MKB_ALLOC(omod, 2 * B * 2 * D * 4);
    MKB_ALLOC(sig, 2 * B * 4);
    MKB_ALLOC(rope, L * 64 * 2 * 4);
    MKB_ALLOC(cfg_lat, size_t(Nmax) * kLatent * 4);
    slots.resize(c.slots);
    for (auto& s : slots) {
        MKB_ALLOC(s.prompt, size_t(Smax) * TD * 4);
        if (!q1) {
            s.kc.resize(NB, nullptr);
            s.vc.resize(NB, nullptr);
            for (int i = 0; i < NB; ++i) {
                MKB_ALLOC(s.kc[i], size_t(H) * Smax * kHeadDim * 2);
                MKB_ALLOC(s.vc[i], size_t(H) * Smax * kHeadDim * 2);
            }
        }
    }
#undef MKB_ALLOC
    return MKB_OK;
}

mkb_status DitImpl::upload_rope(int S, cudaStream_t s)
{
    if (rope_key[0] == S && rope_key[1] == gh && rope_key[2] == gw)
        return MKB_OK;
    const long L = S + long(gh) * gw;
    std::vector<float> t(size_t(L) * kHeadDim);
    const bool q1 = cfg.variant == MKB_VARIANT_QWEN1;
    // Text positions: (t, t, t) in the reference (qwen_image.cpp:136-137); Qwen-Image-1 starts them after the
    // image's centred grid, at max(h/2, w/2). The image takes the frame position S (reference) or 0.
    const long m = q1 ? std::max(gh / 2, gw / 2) : 0;
    for (long i = 0; i < S; ++i)
        rope3(t.data() + i * kHeadDim, m + i, m + i, m + i);
    for (long y = 0; y < gh; ++y)
        for (long x = 0; x < gw; ++x)
            rope3(t.data() + (S + y * gw + x) * kHeadDim, q1 ? 0 : S, y - (gh - gh / 2), x - (gw - gw / 2));
    MKB_TRY_CUDA(cudaMemcpyAsync(rope, t.data(), t.size() * 4, cudaMemcpyHostToDevice, s), "rope upload");
    MKB_TRY_CUDA(cudaStreamSynchronize(s), "rope upload");
    rope_key[0] = S;
    rope_key[1] = gh;
    rope_key[2] = gw;
    return MKB_OK;
}

mkb_status DitImpl::emit(const char* name, int layer, const float* dev, long count, cudaStream_t s)
{
    if (!probe)
        return MKB_OK;
    std::vector<float> h(count);
    MKB_TRY_CUDA(cudaStreamSynchronize(s), "probe sync");
    MKB_TRY_CUDA(cudaMemcpy(h.data(), dev, size_t(count) * 4, cudaMemcpyDeviceToHost), "probe copy");
    probe(name, layer, h.data(), count, probe_user);
    return MKB_OK;
}

mkb_status DitImpl::check_status()
{
    uint32_t v = 0;
    MKB_TRY_CUDA(cudaMemcpy(&v, status, 4, cudaMemcpyDeviceToHost), "status read");
    if (v) {
        cudaMemset(status, 0, 4);
        return fail(MKB_ERR_KERNEL, "dit: kernel status bits 0x" + std::to_string(v));
    }
    return MKB_OK;
}

// Op indices of a plan.
namespace op {
// qwen1: per block 4 ops [qkv, o, ff1, ff2], each the image and text rows in one launch; then globals.
// ref21: per block 4 ops: [qkv, o, gate_up, down]; then globals.
constexpr int kQ1PerBlock = 4, kR21PerBlock = 4;
enum Global { kTxtIn = 0, kImgIn = 1, kProjOut = 2, kTxtIn1 = 3, kCount = 4 };
}  // namespace op

mkb_status DitImpl::build_plan(int B, int S, int N, int first, Plan** out)
{
    const auto key = std::make_tuple(B, S, N, first);
    auto it = plans.find(key);
    if (it != plans.end()) {
        *out = it->second.get();
        return MKB_OK;
    }
    auto plan = std::make_unique<Plan>();
    const bool q1 = cfg.variant == MKB_VARIANT_QWEN1;
    const int L = S + N;
    const char* err = nullptr;
    auto prep = [&](GemmOp& o, Epi epi, const void* X, long ldx, const void* W, long ldw, GemmArgs a,
                    int bn) -> bool {
        a.status = status;
        return gemm_prepare(o, epi, X, ldx, W, ldw, a, bn, &err);
    };
    auto bn_for_pairs = [](const GemmOp& g) { return g.bn >= 128; };
    auto bn_for = [&](int M, int Nc) {
        if (Nc % 256 == 0 && long((M + 127) / 128) * (Nc / 256) >= 74)
            return 256;
        return Nc % 128 == 0 ? 128 : 64;
    };
    const int per = q1 ? op::kQ1PerBlock : op::kR21PerBlock;
    plan->ops.resize(size_t(NB) * per + op::kCount);
    GemmOp* g = plan->ops.data() + size_t(NB) * per;
    if (q1) {
        // This rank's rows (all of them without sequence parallelism): St text and Nl image rows per sample, laid
        // out in the head-major q/k/v buffers as Lh rows per head.
        const SpRows rw = rows_of(S, N);
        const bool sp = sp_world > 1;
        const int St = rw.text, Nl = rw.image, Lh = rw.shard;
        const int Mt = B * St, Mi = B * Nl;
        const long mstride = long(NB) * 12 * D;  // per-sample stride of the stacked modulation
        __nv_bfloat16* xn_s[2] = {xn, xn + size_t(Mt) * D};
        // The O projection's input rows: this GPU's exchange region when peers store into them.
        __nv_bfloat16* const rows_in = sp && sp_heads == 2 ? hx_region_rows(sp_rank) : attn;
        __nv_bfloat16* at_s[2] = {rows_in, rows_in + size_t(Mt) * D};
        __nv_bfloat16* hd_s[2] = {hid, hid + size_t(Mt) * F};
        float* x_s[2] = {x_txt, x_img};
        const int M_s[2] = {Mt, Mi}, rps[2] = {S, Nl}, off[2] = {0, St};
        // RoPE row of head-layout row p: the joint position, p + rank * Lh.
        const float* rope_s[2] = {rope, rope + size_t(sp ? sp_rank : 0) * Lh * kHeadDim};
        // K and V of this rank go straight into its slot of the all-gather buffer, or of the block's K/V buffer of
        // the peer exchange.
        const size_t kv_shard = size_t(B) * H * Lh * kHeadDim;
        auto kv_base = [&](int block) { return sp_p2p ? kv_buf(block & 1) : kv_all; };
        // Head-parallel exchange: Hr heads per rank; span g of the q|k|v buffers holds q, k, v of rank g's heads
        // (hx_chunk elements each), [3][B][Hr][Lh][128].
        const int hx = sp ? sp_heads : 0;
        const int Hr = hx ? H / sp_world : H;
        const size_t hx_chunk = size_t(B) * Hr * Lh * kHeadDim;
        __nv_bfloat16* const hx_recv = hx == 1 ? sp_hx + sp_hx_qkv : hx == 2 ? hx_region_qkv(sp_rank) : nullptr;
        if (hx) {
            HxTables t{};
            const size_t och = size_t(B) * Lh * Hr * kHeadDim;  // mode 1: one output span
            __nv_bfloat16* const o_send = hx == 1 ? hx_recv + sp_hx_qkv : nullptr;
            for (int g = 0; g < sp_world; ++g) {
                const int st_g = g == 0 ? S : 0;  // rank g's text rows
                if (hx == 1) {  // spans to send, this rank's own straight into the receive buffers
                    t.group_dst[g] = (g == sp_rank ? hx_recv : sp_hx) + size_t(g) * 3 * hx_chunk;
                    t.out[g].img = (g == sp_rank ? o_send + sp_hx_o : o_send) + size_t(g) * och;
                } else {  // rank g's receive buffer and input rows, columns of this rank's heads
                    t.group_dst[g] = hx_region_qkv(g) + size_t(sp_rank) * 3 * hx_chunk;
                    __nv_bfloat16* rows = hx_region_rows(g) + size_t(sp_rank) * Hr * kHeadDim;
                    t.out[g].txt = st_g ? rows : nullptr;
                    t.out[g].text_rows = st_g;
                    t.out[g].img = rows + size_t(B) * st_g * D;
                    if (g != sp_rank) {
                        t.sig_qkv[g] = reinterpret_cast<unsigned long long*>(sp_peer[g]) + sp_rank;
                        t.sig_att[g] = reinterpret_cast<unsigned long long*>(sp_peer[g]) + 64 + sp_rank;
                    }
                }
            }
            if (cudaMalloc(&plan->tab, sizeof(HxTables)) != cudaSuccess) {
                cudaGetLastError();
                plan->tab = nullptr;
                return fail(MKB_ERR_ALLOC, "dit: head exchange tables");
            }
            MKB_TRY_CUDA(cudaMemcpy(plan->tab, &t, sizeof(HxTables), cudaMemcpyHostToDevice), "head exchange tables");
        }
        HxTables* const tab = plan->tab;
        const char* nm[2] = {"txt", "img"};
        // Per block four launches, each the image rows' GEMM (problem 0) with the text rows' (problem 1) filling
        // its tail, all on 256 x 256 CTA-pair tiles (QKV: two heads per CTA): the pair halves each SM's W traffic
        // through L2 and shared memory, which is what bounds the 1-CTA tiles (measured fastest for all four at the
        // config-2 shapes).
        for (int i = 0; i < NB; ++i) {
            GemmOp* o = plan->ops.data() + size_t(i) * per;
            for (int s : {1, 0}) {
                if (M_s[s] == 0)  // a sequence-parallel rank other than 0 has no text rows
                    continue;
                const std::string p = "blk" + std::to_string(i) + "." + nm[s] + ".";
                const int stream_idx = s == 0 ? 1 : 0;  // mod order: img then txt per block
                const float* mb = mod + (size_t(i) * 2 + stream_idx) * 6 * D;
                auto put = [&](GemmOp& g, Epi epi, const void* X, long ldx, const void* Wt, long ldw, GemmArgs a,
                               int bn) {
                    if (s == 1)
                        return prep(g, epi, X, ldx, Wt, ldw, a, bn);
                    a.status = status;
                    return gemm_add_problem(g, X, ldx, Wt, ldw, a, &err);
                };
                GemmArgs a;
                a.M = M_s[s];
                a.N = 3 * D;
                a.K = D;
                a.bias = V(p + "qkv.b");
                a.qh = qh;
                a.kh = sp ? kv_base(i) + size_t(sp_rank) * 2 * kv_shard : kh;
                a.vh = sp ? a.kh + kv_shard : vh;
                if (hx) {
                    a.head_group = Hr;
                    a.group_chunk = long(hx_chunk);
                    a.group_dst = reinterpret_cast<__nv_bfloat16* const*>(reinterpret_cast<char*>(tab) +
                                                                          offsetof(HxTables, group_dst));
                }
                a.norm_q = V(p + "norm_q");
                a.norm_k = V(p + "norm_k");
                a.rope = rope_s[s];
                a.D = D;
                a.L = Lh;
                a.seg_rows = rps[s];
                a.seg_off = off[s];
                a.eps = kEps;
                if (!put(o[0], Epi::kQkv, xn_s[s], D, M(p + "qkv.w"), D, a, 256))
                    return fail(MKB_ERR_INVALID, err);
                GemmArgs r;
                r.M = M_s[s];
                r.N = D;
                r.K = D;
                r.bias = V(p + "o.b");
                r.resid = x_s[s];
                r.ldr = D;
                r.gate = mb + 2 * D;
                r.gate_bstride = mstride;
                r.seg_rows = rps[s];
                const int bn_d = D % 256 == 0 ? 256 : 128;
                if (!put(o[1], Epi::kResid, at_s[s], D, M(p + "o.w"), D, r, bn_d))
                    return fail(MKB_ERR_INVALID, err);
                GemmArgs f1;
                f1.M = M_s[s];
                f1.N = F;
                f1.K = D;
                f1.bias = V(p + "ff1.b");
                f1.act = kActGeluTanh;
                f1.out = hd_s[s];
                f1.ldo = F;
                if (!put(o[2], Epi::kBF16, xn_s[s], D, M(p + "ff1.w"), D, f1, F % 256 == 0 ? 256 : 128))
                    return fail(MKB_ERR_INVALID, err);
                GemmArgs f2 = r;
                f2.K = F;
                f2.bias = V(p + "ff2.b");
                f2.gate = mb + 5 * D;
                if (!put(o[3], Epi::kResid, hd_s[s], F, M(p + "ff2.w"), F, f2, bn_d))
                    return fail(MKB_ERR_INVALID, err);
            }
            if (Mi >= 512)
                for (int k = 0; k < 4; ++k)
                    if (bn_for_pairs(o[k]) && !gemm_use_pairs(o[k], &err))
                        return fail(MKB_ERR_INVALID, err);
        }
        GemmArgs a;
        a.M = Mt;
        a.N = D;
        a.K = TD;
        a.bias = V("txt_in.b");
        a.out = x_txt;
        a.ldo = D;
        if (Mt > 0 && !prep(g[op::kTxtIn], Epi::kF32, txt_bf, TD, M("txt_in.w"), TD, a, bn_for(Mt, D)))
            return fail(MKB_ERR_INVALID, err);
        a.M = Mi;
        a.K = kLatent;
        a.bias = V("img_in.b");
        a.out = x_img;
        if (!prep(g[op::kImgIn], Epi::kF32, lat_bf, kLatent, M("img_in.w"), kLatent, a, bn_for(Mi, D)))
            return fail(MKB_ERR_INVALID, err);
        a.N = kLatent;
        a.K = D;
        a.bias = V("proj_out.b");
        a.out = vel;
        a.ldo = kLatent;
        if (!prep(g[op::kProjOut], Epi::kF32, xn + size_t(Mt) * D, D, M("proj_out.w"), D, a, 64))
            return fail(MKB_ERR_INVALID, err);
        // Queries: this rank's Lh rows per head at joint positions rank * Lh...; keys: all L, from the gathered
        // shards when sequence-parallel. Text rows (rank 0) go to the text stream's O input, image rows after them.
        AttnArgs at;
        at.B = B;
        at.H = H;
        at.Lq = Lh;
        at.Lk = L;
        at.q_pos0 = sp ? sp_rank * Lh : 0;
        at.mask = kMaskNone;
        at.scale_log2 = 1.4426950408889634f / std::sqrt(float(kHeadDim));
        at.split = sp && sp_rank > 0 ? sp_rank * Lh : S;
        at.out0 = attn;
        at.ld0 = D;
        at.rows0 = S;
        at.out1 = attn + size_t(Mt) * D;
        at.ld1 = D;
        at.rows1 = Nl;
        if (sp) {
            at.kv_shard_rows = Lh;
            at.kv_plane_stride = 2 * B * H;
        }
        at.status = status;
        if (sp_p2p) {  // shards arrive during the launch; the expected flag value is set per block at launch
            at.own_shard = sp_rank;
            at.shard_ready = reinterpret_cast<const unsigned long long*>(sp_region);
            at.shard_expect = sp_seq + 1;
            if (!attn_prepare(plan->att_odd, qh, Lh, kv_buf(1), kv_buf(1) + kv_shard, L, at, &err))
                return fail(MKB_ERR_INVALID, err);
        }
        if (hx) {  // Hr heads over all L rows, queries and keys in rank shards; outputs to their rows' owners
            at.H = Hr;
            at.Lq = L;
            at.q_pos0 = 0;
            at.q_shard_rows = Lh;
            at.q_plane_stride = 3 * B * Hr;
            at.kv_plane_stride = 3 * B * Hr;
            at.out_shard_rows = Lh;
            at.out_shards = reinterpret_cast<const AttnOutShard*>(reinterpret_cast<char*>(tab) + offsetof(HxTables, out));
            at.ld0 = hx == 1 ? long(Hr) * kHeadDim : D;
            if (hx == 2) {  // peers' rows arrive during the launch; keys in order (the one-GPU rounding)
                at.own_shard = sp_rank;
                at.rotate = 0;
                at.shard_ready = reinterpret_cast<const unsigned long long*>(sp_region);
                at.shard_expect = sp_seq + 1;
            }
            if (!attn_prepare(plan->att, hx_recv, Lh, hx_recv + hx_chunk, hx_recv + 2 * hx_chunk, L, at, &err))
                return fail(MKB_ERR_INVALID, err);
        } else if (!attn_prepare(plan->att, qh, Lh, sp ? kv_base(0) : kh, sp ? kv_base(0) + kv_shard : vh, L, at,
                                 &err))
            return fail(MKB_ERR_INVALID, err);
    } else {
        const int T = first ? L : N, split = first ? S : 0, Mr = B * T;
        const long mstride = 8L * D;  // two modulation rows of 4D per sample
        for (int i = 0; i < NB; ++i) {
            GemmOp* o = plan->ops.data() + size_t(i) * per;
            const std::string p = "blk" + std::to_string(i) + ".";
            GemmArgs a;
            a.M = Mr;
            a.N = 3 * D;
            a.K = D;
            a.qh = qh;
            a.kh = kh;
            a.vh = vh;
            a.norm_q = V(p + "norm_q");
            a.norm_k = V(p + "norm_k");
            a.rope = rope;
            a.D = D;
            a.L = L;
            a.seg_rows = T;
            a.seg_off = first ? 0 : S;
            a.eps = kEps;
            if (!prep(o[0], Epi::kQkv, xn, D, M(p + "qkv.w"), D, a, 256))
                return fail(MKB_ERR_INVALID, err);
            GemmArgs r;
            r.M = Mr;
            r.N = D;
            r.K = D;
            r.resid = x_img;
            r.ldr = D;
            r.gate = mod + D;
            r.gate_bstride = mstride;
            r.seg_rows = T;
            r.tanh_gate = 1;
            r.gate_split = split;
            r.gate_alt_off = 4L * D;
            if (!prep(o[1], Epi::kResid, attn, D, M(p + "o.w"), D, r, bn_for(Mr, D)))
                return fail(MKB_ERR_INVALID, err);
            GemmArgs sg;
            sg.M = Mr;
            sg.N = 2 * F;
            sg.K = D;
            sg.out = hid;
            sg.ldo = F;
            if (!prep(o[2], Epi::kSwiGLU, xn, D, M(p + "gate_up.w"), D, sg, 256))
                return fail(MKB_ERR_INVALID, err);
            GemmArgs r2 = r;
            r2.K = F;
            r2.gate = mod + 3 * D;
            if (!prep(o[3], Epi::kResid, hid, F, M(p + "down.w"), F, r2, bn_for(Mr, D)))
                return fail(MKB_ERR_INVALID, err);
            if (Mr >= 512)
                for (int k = 0; k < 4; ++k)
                    if (bn_for_pairs(o[k]) && !gemm_use_pairs(o[k], &err))
                        return fail(MKB_ERR_INVALID, err);
        }
        GemmArgs a;
        a.M = B * S;
        a.N = D;
        a.K = TD;
        a.act = kActGeluTanh;
        a.out = txt_mid;
        a.ldo = D;
        if (!prep(g[op::kTxtIn1], Epi::kBF16, txt_bf, TD, M("txt_in1.w"), TD, a, bn_for(B * S, D)))
            return fail(MKB_ERR_INVALID, err);
        a.M = Mr;
        a.N = kLatent;
        a.K = D;
        a.act = kActNone;
        a.out = vel;
        a.ldo = kLatent;
        if (!prep(g[op::kProjOut], Epi::kF32, xn, D, M("proj_out.w"), D, a, 64))
            return fail(MKB_ERR_INVALID, err);
        // Per sample: the text input (first step) and the image input into the sample's rows of the joint x.
        plan->per_sample.resize(size_t(B) * 2);
        for (int b = 0; b < B; ++b) {
            GemmArgs t;
            t.M = S;
            t.N = D;
            t.K = D;
            t.out = x_img + size_t(b) * T * D;
            t.ldo = D;
            if (first && !prep(plan->per_sample[2 * b], Epi::kF32, txt_mid + size_t(b) * S * D, D, M("txt_in2.w"), D,
                               t, bn_for(S, D)))
                return fail(MKB_ERR_INVALID, err);
            GemmArgs im;
            im.M = N;
            im.N = D;
            im.K = kLatent;
            im.out = x_img + (size_t(b) * T + split) * D;
            im.ldo = D;
            if (!prep(plan->per_sample[2 * b + 1], Epi::kF32, lat_bf + size_t(b) * N * kLatent, kLatent, M("img_in.w"),
                      kLatent, im, bn_for(N, D)))
                return fail(MKB_ERR_INVALID, err);
        }
        AttnArgs at;
        at.B = B;
        at.H = H;
        at.Lq = T;
        at.Lk = L;
        at.q_pos0 = first ? 0 : S;
        at.q_row0 = first ? 0 : S;
        at.mask = kMaskCondCausal;
        at.cond_len = S;
        at.scale_log2 = 1.4426950408889634f / std::sqrt(float(kHeadDim));
        at.split = S;
        at.out0 = attn;
        at.ld0 = D;
        at.rows0 = T;
        at.out1 = first ? attn + size_t(S) * D : attn;
        at.ld1 = D;
        at.rows1 = T;
        at.status = status;
        if (!attn_prepare(plan->att, qh, L, kh, vh, L, at, &err))
            return fail(MKB_ERR_INVALID, err);
    }
    *out = plan.get();
    plans[key] = std::move(plan);
    return MKB_OK;
}

// The peer exchange's per-step ready values: seq[0] counts steps; block i of step e is announced as e * blocks + i + 1,
// which grows across blocks and steps, so a flag at or above it means that block's shard of this step has landed.
__global__ void k_sp_step(unsigned long long* seq, int blocks)
{
    grid_dep_wait();
    const unsigned long long e = seq[0] + 1;
    seq[0] = e;
    for (int i = 0; i < blocks; ++i)
        seq[1 + i] = e * blocks + i + 1;
    grid_dep_launch();
}

// The head-parallel exchange's returned outputs, src [rank g][sample][shard row][w8 x 8 columns of g's heads], into
// the output projection's input rows (every sample's text rows first, then the image rows), columns g * 8 w8...:
// one 16-byte vector per thread.
__global__ void k_sp_heads_gather(const uint4* __restrict__ src, __nv_bfloat16* __restrict__ attn, int B, int Lh,
                                  int St, int w8, int D, int n)
{
    grid_dep_wait();
    grid_dep_launch();
    const long Mt = long(B) * St;
    for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < n; e += gridDim.x * blockDim.x) {
        const int c = e % w8, rest = e / w8;
        const int i = rest % Lh, gb = rest / Lh;
        const int b = gb % B, g = gb / B;
        const long row = i < St ? long(b) * St + i : Mt + long(b) * (Lh - St) + (i - St);
        reinterpret_cast<uint4*>(attn + row * D + long(g) * w8 * 8)[c] = src[e];
    }
}

// The head exchange over peer memory: raises this rank's flag of the current block (the value at `value`) in every
// peer's region, after everything the kernels before it stored (into the peers' memory too) is complete: the
// dependent-launch wait returns once they are, then a system-scope fence and one release store per peer.
__global__ void k_sp_signal(unsigned long long* const* flags, const unsigned long long* value, int n)
{
    grid_dep_wait();
    const int g = threadIdx.x;
    if (g < n && flags[g]) {
        const unsigned long long v = *value;
        __threadfence_system();
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flags[g]), "l"(v) : "memory");
    }
    grid_dep_launch();
}

// Waits (each lane one peer, bounded like every wait: kErrShardWait on timeout) until every peer's flag in this
// rank's region has reached the current block's value: the peers' attention outputs are in this GPU's rows.
__global__ void k_sp_wait(const unsigned long long* flags, int n, int self, const unsigned long long* value,
                          uint32_t* status)
{
    grid_dep_wait();
    const int g = threadIdx.x;
    if (g < n && g != self)
        wait_flag_ge(flags + g, *value, status, kErrShardWait, nullptr);
    __syncthreads();
    grid_dep_launch();
}

#define MKB_K(expr, what) MKB_TRY_CUDA((expr), what)

// Runs one step for B samples whose latents are in `lat` (device, [B][N][64]) with host noise levels `sigmas`.
// Velocities of sample b's image rows end in vel at rows (b * T + split) (see `first_out` for ref21's layout).
mkb_status DitImpl::run(int B, const int* slot_ids, const float* sigmas, cudaStream_t s, bool* first_out)
{
    if (B < 1 || B > Bmax)
        return fail(MKB_ERR_INVALID, "dit: batch out of range");
    int S = -1, steps = -1;
    for (int b = 0; b < B; ++b) {
        const int id = slot_ids[b];
        if (id < 0 || id >= int(slots.size()) || !slots[id].begun)
            return fail(MKB_ERR_STATE, "dit: step on a slot without begin");
        if (S >= 0 && slots[id].S != S)
            return fail(MKB_ERR_INVALID, "dit: batched slots need the same prompt length");
        if (cfg.variant == MKB_VARIANT_REF21 && steps >= 0 && slots[id].steps != steps)
            return fail(MKB_ERR_INVALID, "dit: batched ref21 slots must be at the same step");
        S = slots[id].S;
        steps = slots[id].steps;
    }
    const int N = gh * gw;
    const bool q1 = cfg.variant == MKB_VARIANT_QWEN1;
    const int first = q1 ? 1 : (steps == 0);
    if (sp_world > 1) {
        SpRows r;
        if (const char* e = sp_partition(S, N, sp_world, sp_rank, &r))
            return fail(MKB_ERR_INVALID, e);
    }
    Plan* plan = nullptr;
    MKB_TRY(upload_rope(S, s));
    MKB_TRY(build_plan(B, S, N, first, &plan));

    // Noise levels of the time path (ref21: rows (sigma, 0) per sample, the image's and the text's).
    const int R = q1 ? B : 2 * B;
    std::vector<float> sv(R);
    for (int b = 0; b < B; ++b) {
        if (q1)
            sv[b] = sigmas[b];
        else {
            sv[2 * b] = sigmas[b];
            sv[2 * b + 1] = 0.0f;
        }
    }
    MKB_K(cudaMemcpyAsync(sig, sv.data(), R * 4, cudaMemcpyHostToDevice, s), "sigma upload");
    if (probe || !use_graphs) {
        MKB_TRY(body(B, slot_ids, S, N, first, plan, s));
    } else {
        std::vector<int> key = {B, S, N, first};
        key.insert(key.end(), slot_ids, slot_ids + B);
        Graph& g = graphs[key];
        if (g.exec) {
            MKB_K(cudaGraphLaunch(g.exec, s), "graph launch");
            count_launch(g.launches);
        } else if (g.seen++ == 0) {
            MKB_TRY(body(B, slot_ids, S, N, first, plan, s));
        } else {
            cudaGraph_t graph = nullptr;
            MKB_K(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
            const unsigned long long l0 = mkb_kernel_launches();
            mkb_status st = body(B, slot_ids, S, N, first, plan, s);
            cudaError_t ce = cudaStreamEndCapture(s, &graph);
            if (st != MKB_OK) {
                if (graph)
                    cudaGraphDestroy(graph);
                return st;
            }
            MKB_K(ce, "end capture");
            g.launches = mkb_kernel_launches() - l0;
            ce = cudaGraphInstantiate(&g.exec, graph, 0);
            cudaGraphDestroy(graph);
            MKB_K(ce, "graph instantiate");
            MKB_K(cudaGraphLaunch(g.exec, s), "graph launch");
        }
    }
    if (!q1)
        for (int b = 0; b < B; ++b)
            slots[slot_ids[b]].steps++;
    if (first_out)
        *first_out = first;
    return MKB_OK;
}

// Everything of a step after the noise levels are on the device: kernel launches only (capturable).
mkb_status DitImpl::body(int B, const int* slot_ids, int S, int N, int first, Plan* plan, cudaStream_t s)
{
    const bool q1 = cfg.variant == MKB_VARIANT_QWEN1;
    const int L = S + N, T = q1 ? L : (first ? L : N), split = q1 ? S : (first ? S : 0);
    const int per = q1 ? op::kQ1PerBlock : op::kR21PerBlock;
    const SpRows rw = rows_of(S, N);  // this rank's text and image rows (all of them unless sequence-parallel)
    const int St = q1 ? rw.text : S, Nl = q1 ? rw.image : N;
    GemmOp* g = plan->ops.data() + size_t(NB) * per;
    const int R = q1 ? B : 2 * B;
    if (sp_p2p || sp_heads == 2) {
        MKB_K(launch_k(k_sp_step, dim3(1), dim3(1), 0, s, sp_seq, NB), "step counter");
        count_launch();
    }
    // Time path: sinusoid -> lin1 -> silu -> lin2 (temb) -> silu -> modulations (qwen_image.cpp:179-205).
    MKB_K(timestep_sinusoid(sig, tp, R, s), "sinusoid");
    MKB_K(gemv(M("time.lin1.w"), tp, kTimeDim, V("time.lin1.b"), h1, D, R, D, kTimeDim, kActSilu, s), "time lin1");
    MKB_K(gemv(M("time.lin2.w"), h1, D, V("time.lin2.b"), temb, D, R, D, D, kActNone, s), "time lin2");
    MKB_TRY(emit("temb", -1, temb, long(R) * D, s));
    MKB_K(silu_f32(temb, st, size_t(R) * D, s), "silu");
    if (q1) {
        // Block 0's modulation on the step's stream, the others on the side stream (joined before their blocks).
        const int Nm = NB * 12 * D;
        MKB_K(gemv(wmat, st, D, wvec, mod, Nm, B, 12 * D, D, kActNone, s), "modulation");
        if (NB > 1) {  // (a fork with no work on the side would leave the step's graph capture unjoined)
            MKB_K(cudaEventRecord(mod_fork, s), "modulation fork");
            MKB_K(cudaStreamWaitEvent(mod_side, mod_fork, 0), "modulation fork");
        }
        for (int i = 1; i < NB; ++i) {
            const size_t r0 = size_t(i) * 12 * D;
            MKB_K(gemv(wmat + r0 * D, st, D, wvec + r0, mod + r0, Nm, B, 12 * D, D, kActNone, mod_side, true),
                  "modulation");
            MKB_K(cudaEventRecord(mod_ready[i], mod_side), "modulation ready");
        }
        MKB_K(gemv(M("norm_out.w"), st, D, V("norm_out.b"), omod, 2 * D, B, 2 * D, D, kActNone, s), "norm_out mod");
    } else {
        MKB_K(gemv(M("mod.w"), st, D, nullptr, mod, 4 * D, R, 4 * D, D, kActNone, s), "modulation");
        MKB_TRY(emit("modulation", -1, mod, long(R) * 4 * D, s));
        MKB_K(gemv(M("norm_out.w"), st, D, nullptr, omod, D, R, D, D, kActNone, s), "norm_out mod");
    }

    // Inputs: text rows (every step for qwen1, the first for ref21) and image rows.
    if (first && St > 0) {
        RmsArgs ra{};
        for (int b = 0; b < B; ++b)
            ra.src[b] = slots[slot_ids[b]].prompt;
        ra.y = txt_bf;
        ra.w = V("txt_norm.w");
        ra.samples = B;
        ra.rows_per_sample = S;
        ra.C = TD;
        ra.eps = kEps;
        MKB_K(rms_norm_rows(ra, s), "txt_norm");
        if (q1) {
            MKB_K(gemm_launch(g[op::kTxtIn], s), "txt_in");
            MKB_TRY(emit("txt_in", -1, x_txt, long(B) * St * D, s));
        } else {
            MKB_K(gemm_launch(g[op::kTxtIn1], s), "txt_in1");
            for (int b = 0; b < B; ++b)
                MKB_K(gemm_launch(plan->per_sample[2 * b], s), "txt_in2");
        }
    }
    MKB_K(cast_f32_bf16(lat, lat_bf, size_t(B) * Nl * kLatent, s), "latents cast");
    if (q1) {
        MKB_K(gemm_launch(g[op::kImgIn], s), "img_in");
        MKB_TRY(emit("img_in", -1, x_img, long(B) * Nl * D, s));
    } else {
        for (int b = 0; b < B; ++b)
            MKB_K(gemm_launch(plan->per_sample[2 * b + 1], s), "img_in");
        MKB_TRY(emit("x_in", -1, x_img, long(B) * T * D, s));
    }

    for (int i = 0; i < NB; ++i) {
        GemmOp* o = plan->ops.data() + size_t(i) * per;
        if (q1) {
            if (i > 0)
                MKB_K(cudaStreamWaitEvent(s, mod_ready[i], 0), "modulation join");
            const int Mt = B * St, Mi = B * Nl;
            const long mstride = long(NB) * 12 * D;
            // The text and image rows' modulated LayerNorms, one launch for both streams.
            auto ln = [&](int scale_off, int shift_off) -> cudaError_t {
                LnModArgs la[2];
                for (int sidx = 0; sidx < 2; ++sidx) {
                    const float* mb = mod + (size_t(i) * 2 + (sidx == 0 ? 1 : 0)) * 6 * D;
                    LnModArgs& l = la[sidx];
                    l = LnModArgs{};
                    l.x = sidx == 0 ? x_txt : x_img;
                    l.y = xn + (sidx == 0 ? 0 : size_t(Mt) * D);
                    l.scale = mb + scale_off * D;
                    l.shift = mb + shift_off * D;
                    l.mod_stride = mstride;
                    l.rows = sidx == 0 ? Mt : Mi;
                    l.D = D;
                    l.rows_per_sample = sidx == 0 ? S : Nl;
                    l.eps = kEps;
                }
                return ln_modulate2(la[0], la[1], s);
            };
            MKB_K(ln(1, 0), "ln_modulate 1");
            if (sp_p2p && i >= 2)  // block i - 2's pushes read the buffer this QKV writes
                for (cudaEvent_t e : sp_done[i & 1])
                    MKB_K(cudaStreamWaitEvent(s, e, 0), "push join");
            MKB_K(gemm_launch(o[0], s), "qkv");
            if (sp_heads == 2) {  // the epilogues store into the peers' memory; flags order the steps
                HxTables* const tab = plan->tab;
                const auto table = [&](size_t off) {
                    return reinterpret_cast<unsigned long long* const*>(reinterpret_cast<char*>(tab) + off);
                };
                const unsigned long long* value = sp_seq + 1 + i;
                MKB_K(launch_k(k_sp_signal, dim3(1), dim3(64), 0, s, table(offsetof(HxTables, sig_qkv)), value,
                               sp_world),
                      "q|k|v stored");
                AttnOp at = plan->att;
                at.args.shard_expect = value;
                MKB_K(attn_launch(at, s), "attention");
                MKB_K(launch_k(k_sp_signal, dim3(1), dim3(64), 0, s, table(offsetof(HxTables, sig_att)), value,
                               sp_world),
                      "outputs stored");
                MKB_K(launch_k(k_sp_wait, dim3(1), dim3(64), 0, s,
                               reinterpret_cast<const unsigned long long*>(sp_region) + 64, sp_world, sp_rank, value,
                               status),
                      "outputs wait");
                count_launch();
                count_launch();
                count_launch();
            } else if (sp_heads) {
                const int Hr = H / sp_world, w8 = Hr * kHeadDim / 8;
                __nv_bfloat16* recv = sp_hx + sp_hx_qkv;
                __nv_bfloat16* o_send = recv + sp_hx_qkv;
                __nv_bfloat16* o_recv = o_send + sp_hx_o;
                MKB_TRY(sp_all_to_all(sp_hx, recv, size_t(3) * B * Hr * rw.shard * kHeadDim, s));
                MKB_K(attn_launch(plan->att, s), "attention");
                MKB_TRY(sp_all_to_all(o_send, o_recv, size_t(B) * rw.shard * Hr * kHeadDim, s));
                const int n = sp_world * B * rw.shard * w8;
                MKB_K(launch_k(k_sp_heads_gather, dim3(std::min((n + 255) / 256, 148 * 8)), dim3(256), 0, s,
                               reinterpret_cast<const uint4*>(o_recv), attn, B, rw.shard, St, w8, D, n),
                      "head gather");
                count_launch();
            } else if (sp_p2p) {
                MKB_TRY(sp_push(B, rw.shard, i, s));
                AttnOp at = i & 1 ? plan->att_odd : plan->att;
                at.args.shard_expect = sp_seq + 1 + i;
                MKB_K(attn_launch(at, s), "attention");
            } else if (sp_world > 1) {  // every rank's K and V shards to every rank, in place
                const size_t count = size_t(2) * B * H * rw.shard * kHeadDim;
                const ncclResult_t r = nccl_api(nullptr)->AllGather(kv_all + size_t(sp_rank) * count, kv_all, count,
                                                                   ncclBfloat16, sp_comm, s);
                if (r != ncclSuccess)
                    return fail(MKB_ERR_CUDA, std::string("dit: K/V all-gather: ") +
                                                  nccl_api(nullptr)->GetErrorString(r));
            }
            if (!sp_p2p && !sp_heads)
                MKB_K(attn_launch(plan->att, s), "attention");
            MKB_K(gemm_launch(o[1], s), "o proj");
            MKB_K(ln(4, 3), "ln_modulate 2");
            MKB_K(gemm_launch(o[2], s), "ff1");
            MKB_K(gemm_launch(o[3], s), "ff2");
            if (probe) {
                MKB_TRY(emit("block.txt", i, x_txt, long(Mt) * D, s));
                MKB_TRY(emit("block.img", i, x_img, long(Mi) * D, s));
            }
        } else {
            const int Mr = B * T;
            LnModArgs la{};
            la.x = x_img;
            la.y = xn;
            la.scale = mod;
            la.shift = nullptr;
            la.mod_stride = 8L * D;
            la.alt_off = 4L * D;
            la.split = split;
            la.rows = Mr;
            la.D = D;
            la.rows_per_sample = T;
            la.eps = kEps;
            MKB_K(ln_modulate(la, s), "ln_modulate 1");
            MKB_K(gemm_launch(o[0], s), "qkv");
            for (int b = 0; b < B; ++b) {
                auto& sl = slots[slot_ids[b]];
                const size_t hoff = size_t(b) * H * L * kHeadDim;
                if (first) {  // keep the text's keys and values (qwen_image.cpp:251-257)
                    MKB_K(copy_head_rows(kh + hoff, L, 0, sl.kc[i], S, 0, H, S, s), "kv save");
                    MKB_K(copy_head_rows(vh + hoff, L, 0, sl.vc[i], S, 0, H, S, s), "kv save");
                } else {  // restore them (qwen_image.cpp:258-262)
                    MKB_K(copy_head_rows(sl.kc[i], S, 0, kh + hoff, L, 0, H, S, s), "kv restore");
                    MKB_K(copy_head_rows(sl.vc[i], S, 0, vh + hoff, L, 0, H, S, s), "kv restore");
                }
            }
            MKB_K(attn_launch(plan->att, s), "attention");
            MKB_K(gemm_launch(o[1], s), "o proj");
            la.scale = mod + 2 * D;
            MKB_K(ln_modulate(la, s), "ln_modulate 2");
            MKB_K(gemm_launch(o[2], s), "gate_up");
            MKB_K(gemm_launch(o[3], s), "down");
            MKB_TRY(emit("block", i, x_img, long(Mr) * D, s));
        }
    }

    if (sp_p2p)  // the last two blocks' pushes
        for (int p = 0; p < 2 && p < NB; ++p)
            for (cudaEvent_t e : sp_done[p])
                MKB_K(cudaStreamWaitEvent(s, e, 0), "push join");

    // norm_out + proj_out (qwen_image.cpp:285-288).
    LnModArgs la{};
    la.D = D;
    la.eps = kEps;
    if (q1) {
        la.x = x_img;
        la.y = xn + size_t(B) * St * D;
        la.scale = omod;
        la.shift = omod + D;
        la.mod_stride = 2L * D;
        la.rows = B * Nl;
        la.rows_per_sample = Nl;
        MKB_K(ln_modulate(la, s), "norm_out");
    } else {
        la.x = x_img;
        la.y = xn;
        la.scale = omod;
        la.mod_stride = 2L * D;
        la.alt_off = D;
        la.split = split;
        la.rows = B * T;
        la.rows_per_sample = T;
        MKB_K(ln_modulate(la, s), "norm_out");
    }
    MKB_K(gemm_launch(g[op::kProjOut], s), "proj_out");
    return MKB_OK;
}

// Latents into `lat`: sample (i * copies + k) takes source sample i's image rows on this rank (all of them unless
// sequence-parallel), for i < n_src and k < copies. Source samples are [N][64] fp32, `kind` says where they live.
mkb_status DitImpl::stage_latents(int n_src, int copies, int S, const float* src, cudaMemcpyKind kind, cudaStream_t s)
{
    const int N = gh * gw;
    const SpRows rw = cfg.variant == MKB_VARIANT_QWEN1 ? rows_of(S, N) : SpRows{S, N, 0, S + N};
    const size_t row = size_t(kLatent) * 4;
    for (int k = 0; k < copies; ++k)
        MKB_K(cudaMemcpy2DAsync(lat + size_t(k) * rw.image * kLatent, copies * rw.image * row,
                                src + size_t(rw.image0) * kLatent, N * row, rw.image * row, n_src, kind, s),
              "latents");
    return MKB_OK;
}

// Sequence-parallel velocities: this rank's image rows of B samples (vel, [B][Nl][64]) into its slot of vel_x at
// their shard positions, an all-gather, then every shard's image rows into out ([B][N][64]).
mkb_status DitImpl::sp_gather_velocity(int B, int S, float* out, cudaMemcpyKind kind, cudaStream_t s)
{
    const int N = gh * gw;
    const SpRows rw = rows_of(S, N);
    const int Lg = rw.shard;
    const size_t row = size_t(kLatent) * 4, slot = size_t(B) * Lg * kLatent;
    MKB_K(cudaMemcpy2DAsync(vel_x + sp_rank * slot + size_t(rw.text) * kLatent, Lg * row, vel, rw.image * row,
                            rw.image * row, B, cudaMemcpyDeviceToDevice, s),
          "velocity exchange");
    const ncclResult_t r = nccl_api(nullptr)->AllGather(vel_x + sp_rank * slot, vel_x, slot, ncclFloat32, sp_comm, s);
    if (r != ncclSuccess)
        return fail(MKB_ERR_CUDA, std::string("dit: velocity all-gather: ") + nccl_api(nullptr)->GetErrorString(r));
    for (int g = 0; g < sp_world; ++g) {
        const int p0 = std::max(g * Lg, S), p1 = (g + 1) * Lg;  // joint rows of shard g that are image rows
        if (p0 >= p1)
            continue;
        MKB_K(cudaMemcpy2DAsync(out + size_t(p0 - S) * kLatent, N * row, vel_x + g * slot + size_t(p0 - g * Lg) * kLatent,
                                Lg * row, (p1 - p0) * row, B, kind, s),
              "velocity exchange");
    }
    return MKB_OK;
}

namespace {

// Device row of reference row r of a gate/up matrix [gate F rows; up F rows], interleaved in blocks of kSwigluBlock.
__host__ __device__ inline long swiglu_row(long r, long F)
{
    const bool up = r >= F;
    const long j = up ? r - F : r;
    return (j / kSwigluBlock) * 2 * kSwigluBlock + (up ? kSwigluBlock : 0) + j % kSwigluBlock;
}

}  // namespace

}  // namespace mkb

struct mkb_dit {
    mkb::DitImpl impl;
};

using namespace mkb;

namespace {

mkb_status check_handle(const mkb_dit* d)
{
    return d ? MKB_OK : fail(MKB_ERR_INVALID, "dit: null handle");
}

// Copies the image rows' velocities of B samples from vel to out_dev (device) on stream s.
mkb_status gather_velocity(DitImpl& m, int B, int S, bool first, float* out, cudaMemcpyKind kind, cudaStream_t s)
{
    if (m.sp_world > 1)
        return m.sp_gather_velocity(B, S, out, kind, s);
    const int N = m.gh * m.gw;
    const bool q1 = m.cfg.variant == MKB_VARIANT_QWEN1;
    const int T = q1 ? N : (first ? S + N : N), split = q1 ? 0 : (first ? S : 0);
    MKB_TRY_CUDA(cudaMemcpy2DAsync(out, size_t(N) * kLatent * 4, m.vel + size_t(split) * kLatent,
                                   size_t(T) * kLatent * 4, size_t(N) * kLatent * 4, B, kind, s),
                 "velocity copy");
    return MKB_OK;
}

}  // namespace

extern "C" {

mkb_status mkb_dit_create(const mkb_dit_config* cfg, mkb_dit** out)
{
    if (!cfg || !out)
        return fail(MKB_ERR_INVALID, "dit_create: null argument");
    auto* d = new (std::nothrow) mkb_dit;
    if (!d)
        return fail(MKB_ERR_ALLOC, "dit_create: host allocation");
    mkb_status s = d->impl.create(*cfg);
    if (s != MKB_OK) {
        delete d;
        return s;
    }
    *out = d;
    return MKB_OK;
}

void mkb_dit_destroy(mkb_dit* d)
{
    if (d) {
        cudaStreamSynchronize(d->impl.stream);
        delete d;
    }
}

mkb_status mkb_dit_init_random(mkb_dit* d, uint64_t seed, float std)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    for (size_t i = 0; i < m.weights.size(); ++i) {
        const Weight& w = m.weights[i];
        const uint64_t key = splitmix64_host(seed * 0x100000001B3ull + i);
        const float sd = w.norm ? 0.1f : std, mean = w.norm ? 1.0f : 0.0f;
        if (w.cols)
            MKB_TRY_CUDA(fill_normal(m.wmat + w.off, true, w.count(), key, 0, sd, mean, m.stream), "init");
        else
            MKB_TRY_CUDA(fill_normal(m.wvec + w.off, false, w.count(), key, 0, sd, mean, m.stream), "init");
    }
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "init sync");
    return MKB_OK;
}

int mkb_dit_weight_count(const mkb_dit* d) { return d ? int(d->impl.weights.size()) : 0; }

mkb_status mkb_dit_weight_info(const mkb_dit* d, int i, const char** name, long* rows, long* cols)
{
    MKB_TRY(check_handle(d));
    if (i < 0 || i >= int(d->impl.weights.size()))
        return fail(MKB_ERR_INVALID, "weight_info: index out of range");
    const Weight& w = d->impl.weights[i];
    if (name)
        *name = w.name.c_str();
    if (rows)
        *rows = w.rows;
    if (cols)
        *cols = w.cols;
    return MKB_OK;
}


int mkb_dit_variant(const mkb_dit* d) { return d ? d->impl.cfg.variant : -1; }

mkb_status mkb_dit_weight_write_rows(mkb_dit* d, const char* name, long row0, long rows, const float* host)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    const Weight* w = name ? m.find(name) : nullptr;
    if (!w || !host)
        return fail(MKB_ERR_INVALID, std::string("weight_write_rows: unknown weight ") + (name ? name : "(null)"));
    if (row0 < 0 || rows <= 0 || row0 + rows > w->rows)
        return fail(MKB_ERR_INVALID, std::string("weight_write_rows: rows out of range for ") + name);
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "sync");
    if (!w->cols) {
        MKB_TRY_CUDA(cudaMemcpy(m.wvec + w->off + row0, host, size_t(rows) * 4, cudaMemcpyHostToDevice),
                     "weight write");
        return MKB_OK;
    }
    std::vector<__nv_bfloat16> tmp(size_t(w->cols));
    for (long r = 0; r < rows; ++r) {
        const long dr = w->swiglu ? swiglu_row(row0 + r, w->rows / 2) : row0 + r;
        for (long c = 0; c < w->cols; ++c)
            tmp[size_t(c)] = __float2bfloat16_rn(host[r * w->cols + c]);
        MKB_TRY_CUDA(cudaMemcpy(m.wmat + w->off + size_t(dr) * w->cols, tmp.data(), size_t(w->cols) * 2,
                                cudaMemcpyHostToDevice),
                     "weight write");
    }
    return MKB_OK;
}

mkb_status mkb_dit_weight_lora_rows(mkb_dit* d, const char* name, long row0, long rows, const float* A,
                                    const float* B, int rank, float scale)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    const Weight* w = name ? m.find(name) : nullptr;
    if (!w || !w->cols || !A || !B)
        return fail(MKB_ERR_INVALID, std::string("lora: unknown matrix ") + (name ? name : "(null)"));
    if (row0 < 0 || rows <= 0 || row0 + rows > w->rows)
        return fail(MKB_ERR_INVALID, std::string("lora: rows out of range for ") + name);
    return lora_merge_rows(m.wmat + w->off, w->cols, row0, rows, w->cols, w->swiglu ? w->rows / 2 : 0, A, B, rank,
                           scale, m.stream);
}

mkb_status mkb_dit_weight_read(mkb_dit* d, const char* name, float* host)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    const Weight* w = name ? m.find(name) : nullptr;
    if (!w || !host)
        return fail(MKB_ERR_INVALID, std::string("weight_read: unknown weight ") + (name ? name : "(null)"));
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "sync");
    if (!w->cols) {
        MKB_TRY_CUDA(cudaMemcpy(host, m.wvec + w->off, w->count() * 4, cudaMemcpyDeviceToHost), "weight read");
        return MKB_OK;
    }
    std::vector<__nv_bfloat16> tmp(w->count());
    MKB_TRY_CUDA(cudaMemcpy(tmp.data(), m.wmat + w->off, w->count() * 2, cudaMemcpyDeviceToHost), "weight read");
    for (long r = 0; r < w->rows; ++r) {
        const long dr = w->swiglu ? swiglu_row(r, w->rows / 2) : r;
        for (long c = 0; c < w->cols; ++c)
            host[r * w->cols + c] = __bfloat162float(tmp[size_t(dr) * w->cols + c]);
    }
    return MKB_OK;
}

mkb_status mkb_dit_weight_write(mkb_dit* d, const char* name, const float* host)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    const Weight* w = name ? m.find(name) : nullptr;
    if (!w || !host)
        return fail(MKB_ERR_INVALID, std::string("weight_write: unknown weight ") + (name ? name : "(null)"));
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "sync");
    if (!w->cols) {
        MKB_TRY_CUDA(cudaMemcpy(m.wvec + w->off, host, w->count() * 4, cudaMemcpyHostToDevice), "weight write");
        return MKB_OK;
    }
    std::vector<__nv_bfloat16> tmp(w->count());
    for (long r = 0; r < w->rows; ++r) {
        const long dr = w->swiglu ? swiglu_row(r, w->rows / 2) : r;
        for (long c = 0; c < w->cols; ++c)
            tmp[size_t(dr) * w->cols + c] = __float2bfloat16_rn(host[r * w->cols + c]);
    }
    MKB_TRY_CUDA(cudaMemcpy(m.wmat + w->off, tmp.data(), w->count() * 2, cudaMemcpyHostToDevice), "weight write");
    return MKB_OK;
}

mkb_status mkb_dit_begin(mkb_dit* d, const float* prompt, int S, int h, int w, int slot)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    if (slot < 0 || slot >= int(m.slots.size()))
        return fail(MKB_ERR_INVALID, "begin: slot out of range");
    if (!prompt || S < 1 || S > m.Smax)
        return fail(MKB_ERR_INVALID, "begin: prompt embeddings must be 1..max_text_tokens rows");
    if (h < 1 || w < 1 || long(h) * w > m.Nmax)
        return fail(MKB_ERR_INVALID, "begin: h * w must be 1..max_image_tokens");
    auto& sl = m.slots[slot];
    MKB_TRY_CUDA(cudaMemcpyAsync(sl.prompt, prompt, size_t(S) * m.TD * 4, cudaMemcpyHostToDevice, m.stream),
                 "prompt upload");
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "prompt upload");
    sl.S = S;
    sl.steps = 0;
    sl.begun = true;
    m.gh = h;
    m.gw = w;
    return MKB_OK;
}

mkb_status mkb_dit_step_batch_dev(mkb_dit* d, int n, const int* slots, const float* latents_dev, const float* sigmas,
                                  float* out_dev, void* stream)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    if (n < 1 || n > m.Bmax || !slots || !latents_dev || !sigmas || !out_dev)
        return fail(MKB_ERR_INVALID, "step: bad arguments");
    if (m.gh * m.gw == 0)
        return fail(MKB_ERR_STATE, "step before begin");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
    for (int i = 0; i < n; ++i)
        if (slots[i] < 0 || slots[i] >= int(m.slots.size()) || !m.slots[slots[i]].begun)
            return fail(MKB_ERR_STATE, "step on a slot without begin");
    bool first = false;
    const int S = m.slots[slots[0]].S;
    MKB_TRY(m.stage_latents(n, 1, S, latents_dev, cudaMemcpyDeviceToDevice, s));
    MKB_TRY(m.run(n, slots, sigmas, s, &first));
    return gather_velocity(m, n, S, first, out_dev, cudaMemcpyDeviceToDevice, s);
}

mkb_status mkb_dit_step_batch(mkb_dit* d, int n, const int* slots, const float* latents, const float* sigmas,
                              float* out)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    if (n < 1 || n > m.Bmax || !slots || !latents || !sigmas || !out)
        return fail(MKB_ERR_INVALID, "step: bad arguments");
    if (m.gh * m.gw == 0)
        return fail(MKB_ERR_STATE, "step before begin");
    for (int i = 0; i < n; ++i)
        if (slots[i] < 0 || slots[i] >= int(m.slots.size()) || !m.slots[slots[i]].begun)
            return fail(MKB_ERR_STATE, "step on a slot without begin");
    bool first = false;
    const int S = m.slots[slots[0]].S;
    MKB_TRY(m.stage_latents(n, 1, S, latents, cudaMemcpyHostToDevice, m.stream));
    MKB_TRY(m.run(n, slots, sigmas, m.stream, &first));
    MKB_TRY(gather_velocity(m, n, S, first, out, cudaMemcpyDeviceToHost, m.stream));
    MKB_TRY_CUDA(cudaStreamSynchronize(m.stream), "step sync");
    return m.check_status();
}

mkb_status mkb_dit_step(mkb_dit* d, const float* latents, float sigma, float* out, int slot)
{
    return mkb_dit_step_batch(d, 1, &slot, latents, &sigma, out);
}

}  // extern "C"

namespace {

// The CFG batch of n_images images (slots 2i / 2i + 1 = cond / uncond) on device latents [n][N][64]; *vel, *T and
// *split locate sample b's velocities at vel + (b * T + split) * 64 (all image rows on every sequence-parallel rank).
mkb_status guided_run(DitImpl& m, int n_images, const float* latents_dev, float sigma, cudaStream_t s,
                      const float** vel, int* T, int* split)
{
    const int B = 2 * n_images;
    if (n_images < 1 || B > m.Bmax || int(m.slots.size()) < B || !latents_dev)
        return fail(MKB_ERR_INVALID, "guided step: need 2 * n_images <= max_batch and as many slots");
    const int N = m.gh * m.gw;
    std::vector<int> ids(B);
    std::vector<float> sg(B, sigma);
    for (int i = 0; i < B; ++i) {
        ids[i] = i;
        if (!m.slots[i].begun)
            return fail(MKB_ERR_STATE, "guided step: slots 0 .. 2 * n_images - 1 need begin");
    }
    const int S = m.slots[0].S;
    // Both predictions of image i see the same latents.
    MKB_TRY(m.stage_latents(n_images, 2, S, latents_dev, cudaMemcpyDeviceToDevice, s));
    bool first = false;
    MKB_TRY(m.run(B, ids.data(), sg.data(), s, &first));
    const bool q1 = m.cfg.variant == MKB_VARIANT_QWEN1;
    *T = q1 ? N : (first ? S + N : N);
    *split = q1 ? 0 : (first ? S : 0);
    *vel = m.vel;
    if (m.sp_world > 1) {  // every rank applies the update to all rows, from the gathered velocities
        MKB_TRY(m.sp_gather_velocity(B, S, m.vel_full, cudaMemcpyDeviceToDevice, s));
        *vel = m.vel_full;
        *T = N;
        *split = 0;
    }
    return MKB_OK;
}

}  // namespace

extern "C" {

mkb_status mkb_dit_step_cfg_dev(mkb_dit* d, int n_images, float* latents_dev, float sigma, float sigma_next,
                                float guidance, void* stream)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
    const float* vel = nullptr;
    int T = 0, split = 0;
    MKB_TRY(guided_run(m, n_images, latents_dev, sigma, s, &vel, &T, &split));
    const size_t img = size_t(m.gh) * m.gw * kLatent;
    for (int i = 0; i < n_images; ++i) {
        const float* vc = vel + (size_t(2 * i) * T + split) * kLatent;
        const float* vu = vel + (size_t(2 * i + 1) * T + split) * kLatent;
        MKB_TRY_CUDA(cfg_euler(latents_dev + i * img, vc, vu, guidance, sigma_next - sigma, img, s), "cfg euler");
    }
    return MKB_OK;
}

mkb_status mkb_dit_guided_velocity_dev(mkb_dit* d, int n_images, const float* latents_dev, float sigma,
                                       float guidance, float* v_out_dev, void* stream)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    if (!v_out_dev)
        return fail(MKB_ERR_INVALID, "guided_velocity: null output");
    cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : m.stream;
    const float* vel = nullptr;
    int T = 0, split = 0;
    MKB_TRY(guided_run(m, n_images, latents_dev, sigma, s, &vel, &T, &split));
    const long img = long(m.gh) * m.gw * kLatent;
    for (int i = 0; i < n_images; ++i)
        MKB_TRY(mkb_cfg_combine_dev(v_out_dev + i * img, vel + (size_t(2 * i) * T + split) * kLatent,
                                    vel + (size_t(2 * i + 1) * T + split) * kLatent, guidance, img, s));
    return MKB_OK;
}

mkb_status mkb_dit_step_cfg(mkb_dit* d, float* latents, float sigma, float sigma_next, float guidance)
{
    MKB_TRY(check_handle(d));
    DitImpl& m = d->impl;
    if (!latents)
        return fail(MKB_ERR_INVALID, "step_cfg: null latents");
    const size_t img = size_t(m.gh) * m.gw * kLatent;
    float* dev = m.cfg_lat;
    mkb_status st = MKB_OK;
    if (cudaMemcpyAsync(dev, latents, img * 4, cudaMemcpyHostToDevice, m.stream) != cudaSuccess)
        st = fail(MKB_ERR_CUDA, "step_cfg: latents upload");
    if (st == MKB_OK)
        st = mkb_dit_step_cfg_dev(d, 1, dev, sigma, sigma_next, guidance, m.stream);
    if (st == MKB_OK && cudaMemcpyAsync(latents, dev, img * 4, cudaMemcpyDeviceToHost, m.stream) != cudaSuccess)
        st = fail(MKB_ERR_CUDA, "step_cfg: latents download");
    if (cudaStreamSynchronize(m.stream) != cudaSuccess && st == MKB_OK)
        st = fail(MKB_ERR_CUDA, "step_cfg: sync");
    if (st == MKB_OK)
        st = m.check_status();
    return st;
}

mkb_status mkb_nccl_unique_id(void* out, size_t bytes)
{
    if (!out || bytes < sizeof(ncclUniqueId))
        return fail(MKB_ERR_INVALID, "nccl_unique_id: need a buffer of MKB_NCCL_ID_BYTES");
    std::string err;
    const NcclApi* api = nccl_api(&err);
    if (!api)
        return fail(MKB_ERR_CUDA, "nccl_unique_id: " + err);
    ncclUniqueId id;
    const ncclResult_t r = api->GetUniqueId(&id);
    if (r != ncclSuccess)
        return fail(MKB_ERR_CUDA, std::string("ncclGetUniqueId: ") + api->GetErrorString(r));
    std::memcpy(out, &id, sizeof(id));
    return MKB_OK;
}

mkb_status mkb_dit_set_sequence_parallel(mkb_dit* d, const void* nccl_id, int rank, int world)
{
    MKB_TRY(check_handle(d));
    return d->impl.set_sp(nccl_id, rank, world);
}

mkb_status mkb_dit_sp_peer_exchange(mkb_dit* d, int enable)
{
    MKB_TRY(check_handle(d));
    return d->impl.sp_set_peer(enable != 0);
}

mkb_status mkb_selftest_peer_wait(const unsigned long long* flags, int n, int self, const unsigned long long* value,
                                  void* stream)
{
    if (!flags || !value || n < 1 || n > 64 || (reinterpret_cast<uintptr_t>(flags) & 7) ||
        (reinterpret_cast<uintptr_t>(value) & 7))
        return fail(MKB_ERR_INVALID, "selftest: need 1-64 8-byte aligned flags and an 8-byte aligned value");
    MKB_TRY_CUDA(launch_k(k_sp_wait, dim3(1), dim3(64), 0, static_cast<cudaStream_t>(stream), flags, n, self, value,
                          device_status_word()),
                 "selftest launch");
    count_launch();
    return MKB_OK;
}

mkb_status mkb_dit_sp_head_exchange(mkb_dit* d, int mode)
{
    MKB_TRY(check_handle(d));
    return d->impl.sp_set_heads(mode);
}

mkb_status mkb_dit_sp_rows(int S, int N, int world, int rank, int* text_rows, int* image_rows, int* image_row0,
                           int* shard_rows)
{
    SpRows r;
    if (const char* e = sp_partition(S, N, world, rank, &r))
        return fail(MKB_ERR_INVALID, e);
    if (text_rows)
        *text_rows = r.text;
    if (image_rows)
        *image_rows = r.image;
    if (image_row0)
        *image_row0 = r.image0;
    if (shard_rows)
        *shard_rows = r.shard;
    return MKB_OK;
}

mkb_status mkb_dit_set_probe(mkb_dit* d, mkb_probe_fn fn, void* user)
{
    MKB_TRY(check_handle(d));
    d->impl.probe = fn;
    d->impl.probe_user = user;
    return MKB_OK;
}

double mkb_dit_step_flops(const mkb_dit* d, int n, int first_step)
{
    if (!d)
        return 0;
    const DitImpl& m = d->impl;
    const double D = m.D, F = m.F, N = double(m.gh) * m.gw;
    double S = 0;
    for (const auto& s : m.slots)
        if (s.begun) {
            S = s.S;
            break;
        }
    const double L = S + N;
    double per;
    if (m.cfg.variant == MKB_VARIANT_QWEN1) {
        per = m.NB * (2 * L * (4 * D * D + 2 * D * F) + 4 * L * L * D);
        per += 2 * S * m.TD * D + 2 * N * 64 * D + 2 * N * D * 64;
    } else {
        const double rows = first_step ? L : N;
        const double att = first_step ? 4 * D * (S * S + N * L) : 4 * D * N * L;
        per = m.NB * (2 * rows * (4 * D * D + 3 * D * F) + att);
        per += (first_step ? 2 * S * (m.TD * D + D * D) : 0) + 2 * N * 64 * D + 2 * rows * D * 64;
    }
    return per * n;
}

}  // extern "C"
