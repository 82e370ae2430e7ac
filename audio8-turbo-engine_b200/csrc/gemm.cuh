// Host-visible pieces of the tcgen05 GEMM (gemm.cu): the epilogue description and the launch plan.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/audio8_b200.h"

namespace a8 {

struct GemmArgs {
  int N, K, M;          // weight rows (output columns), reduction length, token rows
  int ldy;              // output row stride (elements)
  int ntok;             // token tile = UMMA N (multiple of 16, <= 256)
  int n_tiles, tok_tiles;
  int kb_total, kb_per_split, splits;   // splits > 1: the K splits of a tile are one cluster (blockIdx.z = rank)
  int stages;
  uint32_t tmem_cols;
  void* y;
  A8Epilogue epi;
};

struct GemmPlan {
  CUtensorMap tmW, tmX;
  GemmArgs args;
  dim3 grid;
  int smem_bytes;
  int kind;
  bool ok;
};

// Builds the tensor maps and launch shape. Returns 0 or an A8_ERR_* code.
int gemm_plan(GemmPlan* p, const void* x, int ldx, const void* w, int N, int K, int M, void* y, int ldy,
              const A8Epilogue* epi, int splits);
int gemm_launch(const GemmPlan* p, cudaStream_t s, bool pdl);

int encode_map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
                  uint64_t outer, uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle sw);
int encode_map_3d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t d0, uint64_t d1,
                  uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1, uint32_t b2,
                  CUtensorMapSwizzle sw);

}  // namespace a8
