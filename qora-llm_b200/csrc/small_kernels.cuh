// small_kernels.cuh — embedding row lookup, step bookkeeping and Q4 dequantisation.
#pragma once

#include "common.cuh"

namespace qora {

// embed_lookup_q4 (src/gemv.rs:710-736): x[e] = f32(scale) * (q - 8), exact. The table
// is row-interleaved: row v = hidden/2 packed bytes followed by hidden/32 f16 scales.
__global__ void embed_q4_kernel(const uint8_t* table, long long row_bytes, int vocab,
                                int hidden, StepState* st, float* x) {
  const int token = st->token;
  if (token < 0 || token >= vocab) {
    if (threadIdx.x == 0) st->error = 1;
    return;
  }
  const uint8_t* row = table + (long long)token * row_bytes;
  const uint16_t* sc = reinterpret_cast<const uint16_t*>(row + hidden / 2);
  for (int e = threadIdx.x; e < hidden; e += blockDim.x) {
    const uint8_t b = row[e / 2];
    const int q = ((e & 1) ? (b >> 4) : (b & 0xF)) - 8;
    x[e] = __fmul_rn(__half2float(__ushort_as_half(sc[e / kGroup])), (float)q);
  }
}

// End of a decode step: record the greedy token, feed it back, advance the position.
__global__ void advance_kernel(StepState* st, unsigned* ring, int ring_cap) {
  const unsigned a = st->argmax;
  const int s = st->step;
  if (ring && s >= 0 && s < ring_cap) ring[s] = a;
  st->step = s + 1;
  st->token = (int)a;
  st->pos = st->pos + 1;
}

// Rows [row0, row0+rows) of a Q4 [k][n] matrix to f32: (q - 8) * f32(scale).
__global__ void dequant_q4_kernel(const uint8_t* packed, const uint16_t* scales, long long n,
                                  long long row0, long long rows, float* out) {
  const long long total = rows * n;
  const long long gpr = n / kGroup;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const long long r = row0 + i / n, j = i % n;
    const uint8_t b = packed[(r * n + j) / 2];
    const int q = ((j & 1) ? (b >> 4) : (b & 0xF)) - 8;
    const float s = __half2float(__ushort_as_half(scales[r * gpr + j / kGroup]));
    out[i] = __fmul_rn((float)q, s);
  }
}

// Opt-in binary16 KV cache. Host rows [n][row_floats] f32 (token-major, heads h0 .. h0+nh-1
// of the row) -> head-major [nh][head_stride] binary16, rounded to nearest even.
__global__ void kv_pack_f16_kernel(const float* src, int row_floats, int h0, int nh, int n, __half* dst,
                                   long long head_stride) {
  const long long total = (long long)nh * n * kHeadDim;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % kHeadDim);
    const long long t = (i / kHeadDim) % n, h = i / ((long long)kHeadDim * n);
    dst[h * head_stride + t * kHeadDim + d] = __float2half_rn(src[t * row_floats + (h0 + h) * kHeadDim + d]);
  }
}

// The inverse: head-major binary16 -> rows [n][nh*128] f32 (exact).
__global__ void kv_unpack_f16_kernel(const __half* src, long long head_stride, int nh, int n, float* dst) {
  const long long total = (long long)nh * n * kHeadDim;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int d = (int)(i % kHeadDim);
    const long long t = (i / kHeadDim) % n, h = i / ((long long)kHeadDim * n);
    dst[t * nh * kHeadDim + h * kHeadDim + d] = __half2float(src[h * head_stride + t * kHeadDim + d]);
  }
}

}  // namespace qora
