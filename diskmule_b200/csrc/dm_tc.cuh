// dm_tc.cuh -- tcgen05 (5th-generation tensor core) grouped expert GEMM for prefill.
//
// For each (expert, token tile) work item and each 128-row tile of an expert matrix:
//   A = 128 weight rows x K, dequantised by the CTA's threads from GGUF blocks
//       straight to fp16 and stored K-major with the 128-byte swizzle;
//   B = the tile's tokens x K, fp16 (each row scaled by a power of two so large
//       intermediates fit fp16), brought in by TMA with the same swizzle;
//   D = A * B^T accumulated in f32 in tensor memory (TMEM), read back with tcgen05.ld.
// fp16 operands keep the layer within the 1e-3 relative-L2 bar: weights round to
// 2^-11 relative, activations are scaled exactly by powers of two.
#pragma once

#include <cuda.h>

#include "dm_gemv.cuh"

namespace dm {

struct ForwardArgs;

struct TcPlan {
  int nt = 0;          // tokens per tile: 16, 32 or 64
  int max_items = 0;   // grid height bound on (expert, token tile) items
  int rows = 0;        // rows of the packed activation matrices
  __half *x16 = nullptr;   // [rows][H] packed expert inputs (sorted order)
  float *x_inv = nullptr;  // [rows] 1 / scale of each packed input row
  __half *h16 = nullptr;   // [rows][I] packed intermediates
  float *h_inv = nullptr;  // [rows]
  CUtensorMap x_map;       // TMA view of x16: box {64, nt}, 128-byte swizzle
  CUtensorMap h_map;       // TMA view of h16
};

// Whether the tensor-core path covers these formats / shapes.
bool tc_supported(int gate_type, int down_type, int H, int I);

// Encode the two TMA maps for the packed buffers (host, driver entry point).
int make_tc_maps(TcPlan &p, int H, int I, int nt);

// pack -> gate/up -> pack -> down, over the work items built with chunk = p.nt.
int launch_tc_experts(const ForwardArgs &a, const TcPlan &p, const GemvPlan &g,
                      cudaStream_t stream, cudaEvent_t down_mark);

}  // namespace dm
