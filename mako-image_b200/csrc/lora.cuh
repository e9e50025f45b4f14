// LoRA merges into bf16 weight matrices on the device: W[row] += scale * B A for a row range of one matrix.
#pragma once

#include "common.cuh"

#include <cuda_bf16.h>

namespace mkb {

// W: bf16 rows ldw elements apart, logical rows [row0, row0 + rows) of `cols` columns; glu_F > 0 maps logical row r of
// a [2F][cols] gate/up matrix to its device row (two halves interleaved in blocks of 128). A [rank][cols] and
// B [rows][rank] are host fp32 (rank 1..512). Synchronous on `st`.
mkb_status lora_merge_rows(__nv_bfloat16* W, long ldw, long row0, long rows, long cols, long glu_F, const float* A,
                           const float* B, int rank, float scale, cudaStream_t st);

}  // namespace mkb
