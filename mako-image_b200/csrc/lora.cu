#include "lora.cuh"
#include "launch.cuh"

namespace mkb {

namespace {

constexpr int kLoraRows = 16;
constexpr long kGluBlockRows = 128;

__device__ __forceinline__ long glu_device_row(long r, long F)
{
    const bool second = r >= F;
    const long j = second ? r - F : r;
    return (j / kGluBlockRows) * 2 * kGluBlockRows + (second ? kGluBlockRows : 0) + j % kGluBlockRows;
}

// Block (x, y) covers 256 columns of 16 rows: the 16 rows of B sit in shared memory and each A row is read once per
// 16 rows; the sum runs in fp32 and the result is rounded to bf16 once.
__global__ void __launch_bounds__(256) k_lora_merge(__nv_bfloat16* W, long ldw, long row0, int rows, int cols,
                                                     const float* A, const float* Bm, int rank, float scale, long glu_F)
{
    grid_dep_wait();
    grid_dep_launch();
    extern __shared__ float sB[];  // [kLoraRows][rank]
    const int r0 = blockIdx.y * kLoraRows, c = blockIdx.x * 256 + threadIdx.x;
    for (int i = threadIdx.x; i < kLoraRows * rank; i += 256) {
        const int rr = i / rank, k = i - rr * rank;
        sB[i] = r0 + rr < rows ? Bm[long(r0 + rr) * rank + k] : 0.f;
    }
    __syncthreads();
    if (c >= cols)
        return;
    float acc[kLoraRows] = {};
    for (int k = 0; k < rank; ++k) {
        const float a = A[long(k) * cols + c];
#pragma unroll
        for (int rr = 0; rr < kLoraRows; ++rr)
            acc[rr] = fmaf(sB[rr * rank + k], a, acc[rr]);
    }
#pragma unroll
    for (int rr = 0; rr < kLoraRows; ++rr) {
        if (r0 + rr >= rows)
            break;
        const long r = row0 + r0 + rr, dr = glu_F > 0 ? glu_device_row(r, glu_F) : r;
        __nv_bfloat16& w = W[dr * ldw + c];
        w = __float2bfloat16_rn(__bfloat162float(w) + scale * acc[rr]);
    }
}

}  // namespace

mkb_status lora_merge_rows(__nv_bfloat16* W, long ldw, long row0, long rows, long cols, long glu_F, const float* A,
                           const float* B, int rank, float scale, cudaStream_t st)
{
    if (!W || !A || !B || rows <= 0 || cols <= 0 || row0 < 0 || ldw < cols)
        return fail(MKB_ERR_INVALID, "lora: bad arguments");
    if (rank < 1 || rank > 512)
        return fail(MKB_ERR_INVALID, "lora: rank must be 1..512");
    float *dA = nullptr, *dB = nullptr;
    const size_t nA = size_t(rank) * cols, nB = size_t(rows) * rank;
    mkb_status s = MKB_OK;
    if (cudaMalloc(&dA, nA * 4) != cudaSuccess || cudaMalloc(&dB, nB * 4) != cudaSuccess) {
        cudaGetLastError();  // not sticky: keep it out of later launch checks
        s = fail(MKB_ERR_ALLOC, "lora: device staging");
    }
    if (s == MKB_OK && (cudaMemcpyAsync(dA, A, nA * 4, cudaMemcpyHostToDevice, st) != cudaSuccess ||
                        cudaMemcpyAsync(dB, B, nB * 4, cudaMemcpyHostToDevice, st) != cudaSuccess))
        s = fail(MKB_ERR_CUDA, "lora: upload");
    if (s == MKB_OK) {
        const dim3 grid(unsigned((cols + 255) / 256), unsigned((rows + kLoraRows - 1) / kLoraRows));
        launch_k(k_lora_merge, grid, 256, size_t(kLoraRows) * rank * 4, st, W, ldw, row0, int(rows), int(cols), dA,
                 dB, rank, scale, glu_F);
        count_launch();
        s = cuda_status(cudaGetLastError(), "lora merge launch");
    }
    if (cudaStreamSynchronize(st) != cudaSuccess && s == MKB_OK)
        s = fail(MKB_ERR_CUDA, "lora: merge");
    if (dA)
        cudaFree(dA);
    if (dB)
        cudaFree(dB);
    return s;
}

}  // namespace mkb
