// rope.cuh — axial rotary embedding arithmetic, the reference's
// rope_tables_dtype + rope_rotate_half + apply_rope
// (crates/foundry-spike/src/lib.rs:77-129):
//   for axis a (segment [a*dim_a, (a+1)*dim_a)) and j < dim_a/2:
//     f   = pos[a] * theta^(-2j/dim_a)                 (fp32)
//     c,s = cos f, sin f in fp32, rounded to the compute dtype (lib.rs:101-103)
//     y1  = x1*c + (-x2)*s,  y2 = x2*c + x1*s          (x1 = x[j], x2 = x[j+dim_a/2])
// with products and the sum each rounded in fp32 (no fused multiply-add), as
// the reference's separate broadcast_mul and add do. The inverse (gradient of
// apply_rope) is the transposed rotation: x1 = y1*c + y2*s, x2 = y2*c - y1*s.
#pragma once

#include <cuda_bf16.h>
#include <stdint.h>

#include "foundry_attn.h"

namespace fa {

constexpr int kMaxRopeFreqs = 64;  // n_axes * dim_a / 2 for head_dim 128

struct RopeArgs {
  const float* pos;  // (S, n_axes) fp32, nullptr: no rotation
  int n_axes;
  int axis_dim;
  int round_bf16;    // 1: round cos/sin to bf16 (compute dtype bf16)
  int pos_offset;    // token index offset into pos (sequence shards)
  // Optional precomputed (cos, sin) per (token, frequency), tokens indexed
  // like pos (pos_offset applies), n_axes * axis_dim / 2 entries per token,
  // already rounded to the compute dtype. nullptr: evaluate from pos.
  const float2* table;
  // Optional output: a rotation pass that evaluates (cos, sin) itself also
  // writes them here in the table layout (for kernels that run after it).
  float2* table_out;
  float inv_freq[kMaxRopeFreqs];  // theta^(-2j/dim_a), j < dim_a/2
};

// Host: builds the kernel argument block (inv_freq in fp32, correctly rounded
// from double, as the reference's fp32 powf of an exact exponent).
RopeArgs make_rope_args(const fa_rope_t* rope, int round_bf16 = 1,
                        int pos_offset = 0);

__device__ __forceinline__ float round_bf16_f(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// (cos, sin) of frequency f (axis f / half, index f % half) for `token`,
// evaluated from the positions (the table, if any, is not read).
__device__ __forceinline__ float2 rope_cs_direct(const RopeArgs& r, int token, int f) {
  const int t = token + r.pos_offset;
  const int half = r.axis_dim >> 1;
  const float a = __fmul_rn(r.pos[(int64_t)t * r.n_axes + f / half], r.inv_freq[f]);
  float sn, cs;
  sincosf(a, &sn, &cs);
  if (r.round_bf16) {
    cs = round_bf16_f(cs);
    sn = round_bf16_f(sn);
  }
  return make_float2(cs, sn);
}

// The same, from the table when there is one.
__device__ __forceinline__ float2 rope_cs(const RopeArgs& r, int token, int f) {
  if (r.table != nullptr) {
    const int nf = r.n_axes * (r.axis_dim >> 1);
    return r.table[(int64_t)(token + r.pos_offset) * nf + f];
  }
  return rope_cs_direct(r, token, f);
}

// Rotates (inverse == false) or un-rotates one 128-wide row in place.
__device__ __forceinline__ void rope_rotate_row128(const RopeArgs& r,
                                                   int token, float* v,
                                                   bool inverse) {
  const int half = r.axis_dim >> 1;
#pragma unroll 1
  for (int a = 0; a < r.n_axes; ++a) {
    float* seg = v + a * r.axis_dim;
#pragma unroll 4
    for (int j = 0; j < half; ++j) {
      const float2 cs = rope_cs(r, token, a * half + j);
      const float c = cs.x, s = cs.y;
      const float x1 = seg[j];
      const float x2 = seg[j + half];
      if (!inverse) {
        seg[j] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(-x2, s));
        seg[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, s));
      } else {
        seg[j] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
        seg[j + half] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(-x1, s));
      }
    }
  }
}

// Same, for the reference layout (axes of 32 columns covering head_dim 128):
// fully unrolled so the row stays in registers.
__device__ __forceinline__ void rope_rotate_row128_ax32(const RopeArgs& r,
                                                        int token, float* v,
                                                        bool inverse) {
#pragma unroll
  for (int a = 0; a < 4; ++a) {
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const float2 cs = rope_cs(r, token, a * 16 + j);
      const float x1 = v[a * 32 + j];
      const float x2 = v[a * 32 + j + 16];
      if (!inverse) {
        v[a * 32 + j] = __fadd_rn(__fmul_rn(x1, cs.x), __fmul_rn(-x2, cs.y));
        v[a * 32 + j + 16] = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
      } else {
        v[a * 32 + j] = __fadd_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        v[a * 32 + j + 16] = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(-x1, cs.y));
      }
    }
  }
}

}  // namespace fa
