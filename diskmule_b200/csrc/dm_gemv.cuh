// dm_gemv.cuh -- HBM-bound expert GEMV for few tokens per expert (decode).
//
// One thread owns one quant block ("task") of one weight row, issues all of the
// block's 16-byte loads up front, dequantises in registers and applies it to up to
// NT tokens. Partial sums go to shared memory and are reduced per row in a fixed
// order, so results are deterministic.
//
// Nibble -> float without a conversion instruction: PRMT places a quant byte q
// (q < 64) in mantissa bits 16..23 under exponent 0x3F, giving exactly
// f = 0.5 + q/256. Then sum(q*x) = 256 * (sum(f*x) - 0.5*sum(x)), where sum(x) over
// each scale group is precomputed once per token. Block values follow the
// reference's formulas (src/cpu.rs:560-645): Q4_K (d*sc)*q - dmin*m, Q6_K
// (d*sc)*(q-32), Q5_0 d*(q-16), Q8_0 d*q.
#pragma once

#include "dm_common.cuh"

namespace dm {

// Device layouts. Q4_K, BF16, F16 and F32 are read in the reference layout. The
// 2-byte-aligned formats are repacked at layer set-up (a byte permutation):
//   Q6_K -> per block 208 B [ql 128 | qh 64 | scales 16] + f16 d in its own array
//   Q5_0 -> per block 16 B qs, 4 B qh, 2 B d, each in its own array
//   Q8_0 -> per block 32 B qs, 2 B d
struct SplitLayout {
  uint64_t quant_bytes;  // bytes per block in the quant region
  uint64_t qh_bytes;     // bytes per block in the qh region (Q5_0)
};

__host__ __device__ inline SplitLayout split_layout(int kind) {
  switch (kind) {
    case DM_Q6_K: return {208, 0};
    case DM_Q5_0: return {16, 4};
    case DM_Q8_0: return {32, 0};
    default: return {0, 0};
  }
}

// One repacked tensor: `blocks` blocks in [expert][row][block] order.
struct SplitTensor {
  uint8_t *quant = nullptr;  // blocks * quant_bytes
  uint8_t *qh = nullptr;     // blocks * qh_bytes
  uint16_t *d = nullptr;     // blocks
};

int launch_repack(int kind, const uint8_t *src, uint64_t blocks, SplitTensor dst,
                  cudaStream_t stream);

// Per-forward GEMV settings: tokens per pass and the repacked tensors.
struct GemvPlan {
  int nt = 1;          // 1, 2 or 4 tokens per pass over an expert's weights
  int max_active = 0;  // an upper bound on experts with tokens
  int max_items = 0;   // grid height: an upper bound on (expert, chunk) work items
  SplitTensor gate, up, down, sh_gate, sh_up, sh_down;
};

struct ForwardArgs;
// Launch the gate/up (+activation) and down GEMV kernels; `down_mark`, when not
// null, is recorded between them. Returns the number of launches or -1.
int launch_gemv_experts(const ForwardArgs &a, const GemvPlan &plan, cudaStream_t stream,
                        cudaEvent_t down_mark);

}  // namespace dm
