// Fused flash attention on tcgen05 for head dim 64 or 128: softmax(q k^T / sqrt(d)) v over head-major bf16 q/k/v.
// Replaces the runtime's attention() the reference calls per block (src/image/qwen_image.cpp:271), including its
// mask modes, and writes each query row straight into the token-major input of the output projection of its
// stream (text rows and image rows go to separate buffers).
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace mkb {

enum AttnMask : int {
    kMaskNone = 0,      // every query sees every key (Qwen-Image-1 joint attention)
    kMaskCondCausal = 1 // a query at joint position p < cond_len sees keys 0..p (the condition rows are causal, and
                        // never see a later row); queries at p >= cond_len see every key. cond_len = S: the reference's
                        // text rows; cond_len >= Lk: plain causal attention (its CLIP text encoders)
};

struct AttnOutShard {
    __nv_bfloat16* txt = nullptr;
    __nv_bfloat16* img = nullptr;
    int text_rows = 0;
    int pad = 0;
};

struct AttnArgs {
    int B = 0, H = 0;
    int Lq = 0;          // query rows per (sample, head) in q
    int Lk = 0;          // key rows per (sample, head) in k / v
    int q_pos0 = 0;      // joint position of query row 0 (keys start at joint position 0)
    int q_row0 = 0;      // row of q (within each head) holding query row 0
    int mask = kMaskNone;
    int cond_len = 0;    // kMaskCondCausal boundary
    float scale_log2 = 0.f;  // softmax scale * log2(e)
    int head_dim = 128;      // 64 or 128
    // Output routing by joint position p of a query row: p < split -> out0 row (b * rows0 + p),
    // else out1 row (b * rows1 + p - split); columns [h * 128, h * 128 + 128).
    int split = 0;
    __nv_bfloat16* out0 = nullptr;
    long ld0 = 0;
    int rows0 = 0;
    __nv_bfloat16* out1 = nullptr;
    long ld1 = 0;
    int rows1 = 0;
    // Keys and values split into shards of kv_shard_rows rows (a multiple of 128; 0 = one unsplit [B*H][Lk] plane
    // per head): key row j of head bh is row j % kv_shard_rows of plane (j / kv_shard_rows) * kv_plane_stride + bh
    // of the k / v maps. This is the layout a sequence-parallel all-gather leaves (one shard per rank).
    int kv_shard_rows = 0;
    int kv_plane_stride = 0;
    // Queries split the same way (q_shard_rows a multiple of 128, 0 = unsplit; needs q_row0 = 0): query row r of
    // head bh is row r % q_shard_rows of plane (r / q_shard_rows) * q_plane_stride + bh of the q map.
    int q_shard_rows = 0;
    int q_plane_stride = 0;
    // Outputs by shards of out_shard_rows joint positions (0 = the split routing above): position p of sample b
    // is local row i = p % out_shard_rows of shard g = p / out_shard_rows and goes through out_shards[g] (a device
    // array, one entry per shard): i < text_rows to row (b * text_rows + i) of txt, else to row
    // (b * (out_shard_rows - text_rows) + i - text_rows) of img; rows ld0 apart, columns [h * head_dim, ...). The
    // head-parallel exchange's destinations, one per owning rank (its send span, or its rows on that GPU).
    int out_shard_rows = 0;
    const AttnOutShard* out_shards = nullptr;
    // Shards that other ranks copy in while the kernel runs (the peer-memory K/V exchange). own_shard >= 0 makes
    // every CTA take its key tiles starting with shard own_shard (written on this GPU before the launch) and
    // wrapping round, and wait before the first tile of any other shard g until shard_ready[g] >= *shard_expect
    // (an acquire load at system scope, bounded by kWaitNs; on timeout the kErrShardWait bit). Needs
    // kv_shard_rows > 0 and kMaskNone. The key order only changes the online softmax's rounding. rotate = 0 keeps
    // the keys in order (shard 0 first: the one-GPU rounding), with the same waits before every shard other than
    // the last one confirmed; query tiles of a shard other than own_shard (q_shard_rows > 0) wait the same way
    // before they are loaded. The head-parallel exchange over peer memory, whose peers store q, k and v here.
    int own_shard = -1;
    int rotate = 1;
    const unsigned long long* shard_ready = nullptr;
    const unsigned long long* shard_expect = nullptr;
    uint32_t* status = nullptr;
};

struct AttnOp {
    CUtensorMap tq, tk, tv;
    AttnArgs args;
    dim3 grid;
    bool pair = false;  // CTA pairs (head dim 128): K read in 64-row halves, grid.x even
    bool ready = false;
};

// Single-head attention at head dim d = 256 or 512 over n rows whose q, k and v sit side by side in one bf16 buffer
// (rows of ld elements; q, k, v at columns q_col, k_col, v_col): out[row][0, d) = softmax(q k^T / sqrt(d)) v, bf16,
// rows ldo apart (the VAE decoder's mid-block attention, Engine::vae_attention, src/image/engine.cpp:748-778).
struct AttnWideArgs {
    int n = 0, d = 0;
    int q_col = 0, k_col = 0, v_col = 0;
    __nv_bfloat16* out = nullptr;
    long ldo = 0;
    float scale_log2 = 0.f;  // softmax scale * log2(e)
    uint32_t* status = nullptr;
};

struct AttnWideOp {
    CUtensorMap tm;
    AttnWideArgs args;
    dim3 grid;
    bool ready = false;
};

bool attn_wide_prepare(AttnWideOp& op, const void* qkv, long ld, const AttnWideArgs& args, const char** err);
cudaError_t attn_wide_launch(const AttnWideOp& op, cudaStream_t stream);

// q: [B][H][Lq_rows][d], k/v: [B][H][Lk_rows][d] (bf16, contiguous); Lq_rows >= args.Lq, Lk_rows >= args.Lk.
bool attn_prepare(AttnOp& op, const void* q, int Lq_rows, const void* k, const void* v, int Lk_rows,
                  const AttnArgs& args, const char** err);
cudaError_t attn_launch(const AttnOp& op, cudaStream_t stream);

}  // namespace mkb
