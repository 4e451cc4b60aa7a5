// common.cuh — shared device helpers for the sm_100a decode engine.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define QORA_DEV __device__ __forceinline__

namespace qora {

constexpr int kGroup = 32;      // Q4 group size along the output dim (src/gemv.rs:20)
constexpr int kHeadDim = 128;   // SmolLM3 head_dim (src/main.rs:102)
constexpr int kHalfDim = 64;

// Decode-step state kept in device memory so that one captured CUDA graph serves every
// step: the graph's kernels read the position and token from here.
struct StepState {
  int pos;       // KV rows already filled; this step appends row `pos`
  int token;     // input token id of this step
  unsigned argmax;  // greedy result of this step
  int step;      // index into the generation output ring
  int error;     // nonzero: a kernel rejected its input (bad token id)
  int pad[3];
};

QORA_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

QORA_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Block-wide sum of one float per thread; result broadcast to all threads. `red` must
// hold blockDim.x/32 floats. Ends with a __syncthreads so `red` can be reused.
QORA_DEV float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = 0.0f;
  for (int w = 0; w < nw; ++w) t += red[w];  // fixed order: deterministic
  __syncthreads();
  return t;
}

// RMSNorm scale 1 / sqrt(mean(x^2) + 1e-6) (rms_norm_f16, src/gemv.rs:744-747).
QORA_DEV float rms_inv(const float* x, int n, float* red) {
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) s = __fmaf_rn(x[i], x[i], s);
  const float tot = block_sum(s, red);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)n), 1e-6f)));
}

// Greedy comparison: larger value wins, equal values go to the lower index (the first
// strict maximum of src/generate.rs:349-351). NaN never wins.
QORA_DEV bool better(float v, unsigned i, float bv, unsigned bi) {
  return v > bv || (v == bv && i < bi);
}

}  // namespace qora
