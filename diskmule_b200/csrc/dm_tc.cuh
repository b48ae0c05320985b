// dm_tc.cuh -- tcgen05 (5th-generation tensor core) grouped expert GEMM for prefill.
//
// One persistent CTA per SM walks work units (expert token tile x 128-row weight tile).
// For each 256-wide K step of a unit:
//   A = 128 weight rows: the raw GGUF blocks of the step arrive by TMA in a ring of
//       shared-memory stages, are dequantised in f32 by the producer warps, rounded once
//       to fp16 and written straight into tensor memory (TMEM) with tcgen05.st;
//   B = the tile's tokens, fp16 (each row scaled by a power of two, optionally split
//       into hi + lo halves), brought into shared memory by TMA with the 128-byte swizzle;
//   D = A * B^T accumulated in f32 in TMEM (two accumulators, so the epilogue of one
//       unit overlaps the next unit's MMAs) and read back with tcgen05.ld.
// fp16 operands keep the layer within the 1e-3 relative-L2 bar: weights round to
// 2^-11 relative, activations are scaled exactly by powers of two.
#pragma once

#include <cuda.h>

#include "dm_gemv.cuh"

namespace dm {

struct ForwardArgs;

struct TcWeights;

struct TcPlan {
  const TcWeights *weights = nullptr;  // the layer's weight views
  int nt = 0;          // tokens per tile: 16, 32 or 64
  int max_items = 0;   // grid height bound on (expert, token tile) items
  int rows = 0;        // rows of the packed activation matrices
  int n_sm = 148;      // persistent grid size
  bool split = true;   // B as hi + lo fp16 halves where shared memory allows:
  bool split_x = true, split_h = true;  // as encoded for the inputs / intermediates
  bool bf16 = false;   // bf16 weights: gathered bf16 inputs, bf16 hi/lo intermediates
  __half *x16 = nullptr;   // [rows][H] packed expert inputs (sorted order)
  float *x_inv = nullptr;  // [rows] 1 / scale of each packed input row
  __half *h16 = nullptr;   // [rows][I] packed intermediates
  float *h_inv = nullptr;  // [rows]
  float *gu = nullptr;     // [rows][2I] gate/up outputs (gate i at 2i, up i at 2i + 1)
  CUtensorMap x_map;       // TMA view of x16: box {64, nb, 4 atoms}, 128-byte swizzle
  CUtensorMap h_map;       // TMA view of h16
  CUtensorMap h1_map;      // bf16 layers: h16 as single fp16 rows [rows][I] (f16 down path)
  CUtensorMap x_map_pair, h1_map_pair;  // the same with 128-row boxes (CTA-pair kernels)
};

// Device-side pointers of the per-step transposed down arrays (see TcWeights).
struct TcSide {
  const uint8_t *qh_t = nullptr, *d_t = nullptr;        // routed experts
  const uint8_t *sh_qh_t = nullptr, *sh_d_t = nullptr;  // shared expert
  int up_swapped = 0, sh_up_swapped = 0;  // 1: index 0 of the gate|up axis is `up`
  // bf16 layers: the largest L2 norm of a gate row / an up row of each expert (index E:
  // the shared expert), or null
  const float *gate_norm = nullptr, *up_norm = nullptr;
};

// Per-layer tensor-core views of the expert weights, built once.
struct TcWeights {
  CUtensorMap up, sh_up;      // Q4_K gate/up: {row bytes, gate|up, row, expert},
                              // box {144, 2, 64, 1} = 64 interleaved gate/up row pairs
  CUtensorMap down, sh_down;  // down quant bytes: {row bytes, expert*H + row}, box {., 128}
  CUtensorMap down16, sh_down16;  // bf16 layers: fp16 copies of the down weights
  bool f16_down = false;          // bf16 layers: down product on fp16 copies (one MMA per step)
  TcSide side;
};

// Bytes of the per-step transposed down arrays: Q6_K d, or Q5_0 qh and d.
void tc_side_bytes(int down_type, uint64_t experts, int H, int I, uint64_t *qh_bytes,
                   uint64_t *d_bytes);

// Encode the weight maps and fill the side arrays (preallocated: qh_t/d_t for the routed
// experts, sh_qh_t/sh_d_t for the shared one). Returns 0 or -1 when a map is refused.
int make_tc_weights(TcWeights &w, const uint8_t *gate, const uint8_t *up, uint64_t expert_stride,
                    const uint8_t *sh_gate, const uint8_t *sh_up, const SplitTensor &down,
                    const SplitTensor &sh_down, int down_type, int experts, int H, int I,
                    uint8_t *qh_t, uint8_t *d_t, uint8_t *sh_qh_t, uint8_t *sh_d_t,
                    cudaStream_t stream);

// bf16 weights (no side arrays): gate/up {K, gate|up, row, expert}, down {K, expert*H + row}.
// down16 / sh_down16, when given, are fp16 copies of the down weights (same layout): the
// down product then runs on them with single fp16 intermediates.
int make_tc_weights_bf16(TcWeights &w, const uint8_t *gate, const uint8_t *up, uint64_t expert_stride,
                         const uint8_t *sh_gate, const uint8_t *sh_up, const uint8_t *down,
                         const uint8_t *sh_down, int experts, int H, int I,
                         const uint8_t *down16 = nullptr, const uint8_t *sh_down16 = nullptr);

// out[e] = max(out[e], largest L2 norm of the `rows` bf16 rows of K elements of expert e),
// experts `expert_stride` bytes apart (layer set-up; out starts at zero).
void launch_row_norm_max(const void *w, uint64_t expert_stride, int experts, int rows, int K,
                         float *out, cudaStream_t stream);

// bf16 -> fp16 copy of n elements (exact for magnitudes in fp16's normal range, 2^-14 to
// 65504; smaller ones round to fp16's subnormal grid of 2^-24).
void launch_bf16_to_f16(const void *src, void *dst, uint64_t n, cudaStream_t stream);

// Whether the tensor-core path covers these formats / shapes.
bool tc_supported(int gate_type, int down_type, int H, int I);

// Decide the split per matrix and encode the two TMA maps for the packed buffers
// (host, driver entry point).
int make_tc_maps(TcPlan &p, int H, int I, int down_type, int nt);

// pack -> gate/up -> pack -> down, over the work items built with chunk = p.nt.
int launch_tc_experts(const ForwardArgs &a, const TcPlan &p, const TcWeights &w,
                      cudaStream_t stream, cudaEvent_t down_mark);

// One thread waits, bounded by `cycles`, on a barrier nothing arrives on; *status gets
// kStatusTimeout (a self-test of the kernels' bounded waits).
void launch_selftest_wait(long long cycles, int32_t *status, cudaStream_t s);

}  // namespace dm
