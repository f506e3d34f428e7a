// qk_prologue.cu — the joint block's q/k prologue, fused: per stream RMSNorm
// over the head dim, the axial RoPE, and the text-then-image concatenation.
//
// Reference (crates/foundry-spike/src/lib.rs): rms_norm (:45-58; statistics
// in fp32, x / sqrt(mean(x^2) + eps) cast to the compute dtype, times the
// weight in that dtype), apply_rope (:122-129) with the tables of
// rope_tables_dtype (:77-105), applied per stream with its own q/k norm
// weight (:326-358), then cat([txt, img]) (:363-365). Here one pass reads the
// two streams' projections through their own strides and writes the joint
// rotated (B, T+I, H, 128) tensor the attention kernels read; the backward
// pass maps the joint gradient back through the rotation and the RMSNorm to
// the two streams and accumulates the norm weights' gradients.
//
// Layout of the work: eight consecutive joint tokens per block (all heads);
// a half-warp owns one (token, head) row, lane l elements 8l..8l+7 (16-byte
// accesses); the rotate-half partner of element 8l+u is element 8(l^2)+u.
#include <cuda_bf16.h>

#include "attn_common.h"
#include "rope.cuh"
#include "sm100_ptx.cuh"

namespace fa {
namespace qkp {

constexpr int kTokens = 8;
constexpr int kThreads = 256;
constexpr int kMaxRows = 12;  // rows per half-warp: 8 tokens x H, H <= 24

// strided (B, S, H, 128) view: element strides, head dim contiguous
struct View {
  void* p;
  int64_t sb, ss, sh;
};

struct Seg {
  const __nv_bfloat16* x;  // stream tensor (B, len, H, 128)
  int64_t sb, ss, sh;
  const __nv_bfloat16* w;  // (128,) norm weight
};

__device__ __forceinline__ void unpack8(const uint4& v, float* e) {
  e[0] = __uint_as_float(v.x << 16); e[1] = __uint_as_float(v.x & 0xFFFF0000u);
  e[2] = __uint_as_float(v.y << 16); e[3] = __uint_as_float(v.y & 0xFFFF0000u);
  e[4] = __uint_as_float(v.z << 16); e[5] = __uint_as_float(v.z & 0xFFFF0000u);
  e[6] = __uint_as_float(v.w << 16); e[7] = __uint_as_float(v.w & 0xFFFF0000u);
}

__device__ __forceinline__ uint4 pack8(const float* e) {
  return make_uint4(pack_bf16(e[0], e[1]), pack_bf16(e[2], e[3]), pack_bf16(e[4], e[5]),
                    pack_bf16(e[6], e[7]));
}

__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// sum over the 16 lanes of a half-warp (all 32 lanes take part)
__device__ __forceinline__ float half_warp_sum(float v) {
#pragma unroll
  for (int off = 8; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Joint row (token s, head h) -> its stream's element pointer (lane offset added).
__device__ __forceinline__ const __nv_bfloat16* src_row(const Seg& txt, const Seg& img, int T,
                                                        int b, int s, int h, int l) {
  const Seg& g = s < T ? txt : img;
  const int ls = s < T ? s : s - T;
  return g.x + b * g.sb + (int64_t)ls * g.ss + h * g.sh + 8 * l;
}

__global__ void __launch_bounds__(kThreads, 2)
qk_norm_rope_fwd_kernel(Seg txt, Seg img, int T, int S, int H, float eps,
                        const __grid_constant__ RopeArgs r, View y) {
  __shared__ float2 cs_s[kTokens][64];
  __shared__ float w_s[2][128];
  const int tiles = (S + kTokens - 1) / kTokens;
  const int s0 = (int)(blockIdx.x % tiles) * kTokens, b = (int)(blockIdx.x / tiles);
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int rows = kTokens * H;
  const bool rotate = r.pos != nullptr;
  uint4 v[kMaxRows];
#pragma unroll
  for (int k = 0; k < kMaxRows; ++k) {
    const int row = hw + k * (kThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    v[k] = make_uint4(0, 0, 0, 0);
    if (row < rows && s < S)
      v[k] = *reinterpret_cast<const uint4*>(src_row(txt, img, T, b, s, h, l));
  }
  if (rotate) {
    for (int i = threadIdx.x; i < kTokens * 64; i += kThreads) {
      const int t = i >> 6, f = i & 63, s = s0 + t;
      if (s < S) cs_s[t][f] = rope_cs(r, s, f);
    }
  }
  // the two streams' norm weights (no weights: no normalisation, the rows
  // are only rotated and concatenated)
  const bool norm = txt.w != nullptr;
  if (norm)
    for (int i = threadIdx.x; i < 2 * 128; i += kThreads)
      w_s[i >> 7][i & 127] = __bfloat162float((i >> 7 ? img.w : txt.w)[i & 127]);
  __syncthreads();
  const bool first = (l & 3) < 2;  // element in the first half of its axis
  const float sgn = first ? -1.f : 1.f;
  const int f0 = (l >> 2) * 16 + (l & 1) * 8;
#pragma unroll
  for (int k = 0; k < kMaxRows; ++k) {
    const int row = hw + k * (kThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    const bool live = row < rows && s < S;  // uniform per half-warp
    float e[8];
    unpack8(v[k], e);
    if (norm) {
      float ss = 0.f;
#pragma unroll
      for (int u = 0; u < 8; ++u) ss = fmaf(e[u], e[u], ss);
      ss = half_warp_sum(ss);
      const float scale = sqrtf(ss / 128.f + eps);
      const float* w = &w_s[s < T ? 0 : 1][8 * l];
#pragma unroll
      for (int u = 0; u < 8; ++u) e[u] = round_bf16(round_bf16(e[u] / scale) * w[u]);
    }
    if (rotate) {
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = __shfl_xor_sync(0xffffffffu, e[u], 2);
      if (live) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float2 c = cs_s[t][f0 + u];
          e[u] = __fadd_rn(__fmul_rn(e[u], c.x), __fmul_rn(sgn * o[u], c.y));
        }
      }
    }
    if (live)
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(y.p) + b * y.sb +
                                (int64_t)s * y.ss + h * y.sh + 8 * l) = pack8(e);
  }
}

__global__ void __launch_bounds__(kThreads, 1)
qk_norm_rope_bwd_kernel(Seg txt, Seg img, int T, int S, int H, float eps,
                        const __grid_constant__ RopeArgs r, View dy, View dx_txt, View dx_img,
                        float* dw_txt, float* dw_img) {
  __shared__ float2 cs_s[kTokens][64];
  __shared__ float dw_s[2][128];
  __shared__ float w_s[2][128];
  const int tiles = (S + kTokens - 1) / kTokens;
  const int s0 = (int)(blockIdx.x % tiles) * kTokens, b = (int)(blockIdx.x / tiles);
  const int hw = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int rows = kTokens * H;
  const bool rotate = r.pos != nullptr;
  uint4 xv[kMaxRows], gv[kMaxRows];
#pragma unroll
  for (int k = 0; k < kMaxRows; ++k) {
    const int row = hw + k * (kThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    xv[k] = make_uint4(0, 0, 0, 0);
    gv[k] = make_uint4(0, 0, 0, 0);
    if (row < rows && s < S) {
      xv[k] = *reinterpret_cast<const uint4*>(src_row(txt, img, T, b, s, h, l));
      gv[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(dy.p) +
                                               b * dy.sb + (int64_t)s * dy.ss + h * dy.sh + 8 * l);
    }
  }
  for (int i = threadIdx.x; i < 2 * 128; i += kThreads) dw_s[i >> 7][i & 127] = 0.f;
  if (rotate) {
    for (int i = threadIdx.x; i < kTokens * 64; i += kThreads) {
      const int t = i >> 6, f = i & 63, s = s0 + t;
      if (s < S) cs_s[t][f] = rope_cs(r, s, f);
    }
  }
  const bool norm = txt.w != nullptr;
  if (norm)
    for (int i = threadIdx.x; i < 2 * 128; i += kThreads)
      w_s[i >> 7][i & 127] = __bfloat162float((i >> 7 ? img.w : txt.w)[i & 127]);
  __syncthreads();
  // the transposed rotation: g = dy*c + rot^T(dy*s), rot^T([a|b]) = [b|-a]
  const bool first = (l & 3) < 2;
  const float sgn = first ? 1.f : -1.f;
  const int f0 = (l >> 2) * 16 + (l & 1) * 8;
#pragma unroll
  for (int k = 0; k < kMaxRows; ++k) {
    const int row = hw + k * (kThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    const bool live = row < rows && s < S;
    float x[8], g[8];
    unpack8(xv[k], x);
    unpack8(gv[k], g);
    if (rotate) {
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = __shfl_xor_sync(0xffffffffu, g[u], 2);
      if (live) {
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float2 c = cs_s[t][f0 + u];
          g[u] = round_bf16(__fadd_rn(__fmul_rn(g[u], c.x), __fmul_rn(sgn * o[u], c.y)));
        }
      }
    }
    const bool is_txt = s < T;
    if (!norm) {  // rotation and concatenation only: dx is the un-rotated gradient
      if (live) {
        const View& dx = is_txt ? dx_txt : dx_img;
        const int ls = is_txt ? s : s - T;
        *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dx.p) + b * dx.sb +
                                  (int64_t)ls * dx.ss + h * dx.sh + 8 * l) = pack8(g);
      }
      continue;
    }
    // statistics of the forward, recomputed from x
    float ss = 0.f;
#pragma unroll
    for (int u = 0; u < 8; ++u) ss = fmaf(x[u], x[u], ss);
    ss = half_warp_sum(ss);
    const float scale = sqrtf(ss / 128.f + eps);
    const float* w = &w_s[is_txt ? 0 : 1][8 * l];
    float gn[8], dot = 0.f;
    float* dws = &dw_s[is_txt ? 0 : 1][8 * l];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const float n = round_bf16(x[u] / scale);
      if (live) atomicAdd(dws + u, g[u] * n);  // the weights' gradient: block partials
      gn[u] = round_bf16(g[u] * w[u]);
      dot = fmaf(gn[u], x[u], dot);
    }
    dot = half_warp_sum(dot);
    const float k3 = dot / (128.f * scale * scale * scale);
    float d[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) d[u] = gn[u] / scale - x[u] * k3;
    if (live) {
      const View& dx = is_txt ? dx_txt : dx_img;
      const int ls = is_txt ? s : s - T;
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(dx.p) + b * dx.sb +
                                (int64_t)ls * dx.ss + h * dx.sh + 8 * l) = pack8(d);
    }
  }
  // weight gradients: one global add per column and stream of the block's
  // partial sums
  __syncthreads();
  for (int i = threadIdx.x; i < 2 * 128; i += kThreads) {
    float* dst = (i >> 7) == 0 ? dw_txt : dw_img;
    const float v = dw_s[i >> 7][i & 127];
    if (dst != nullptr && v != 0.f) atomicAdd(dst + (i & 127), v);
  }
}

}  // namespace qkp

static qkp::Seg make_seg(const fa_tensor_t* x, const void* w) {
  qkp::Seg g;
  g.x = x ? reinterpret_cast<const __nv_bfloat16*>(x->data) : nullptr;
  g.sb = x ? x->stride_b : 0;
  g.ss = x ? x->stride_s : 0;
  g.sh = x ? x->stride_h : 0;
  g.w = reinterpret_cast<const __nv_bfloat16*>(w);
  return g;
}

int launch_qk_norm_rope_fwd(int B, int T, int I, int H, const fa_tensor_t* x_txt,
                            const fa_tensor_t* x_img, const void* w_txt, const void* w_img,
                            float eps, const fa_rope_t* rope, const fa_tensor_t* y,
                            cudaStream_t stream) {
  const int S = T + I;
  // a stream of length 0 is stood in for by the other (its rows never occur)
  const qkp::Seg txt = T > 0 ? make_seg(x_txt, w_txt) : make_seg(x_img, w_img);
  const qkp::Seg img = I > 0 ? make_seg(x_img, w_img) : txt;
  const RopeArgs r = make_rope_args(rope, 1, 0);
  const int tiles = (S + qkp::kTokens - 1) / qkp::kTokens;
  qkp::qk_norm_rope_fwd_kernel<<<(unsigned)((int64_t)B * tiles), qkp::kThreads, 0, stream>>>(
      txt, img, T, S, H, eps, r, qkp::View{y->data, y->stride_b, y->stride_s, y->stride_h});
  return launch_status();
}

int launch_qk_norm_rope_bwd(int B, int T, int I, int H, const fa_tensor_t* x_txt,
                            const fa_tensor_t* x_img, const void* w_txt, const void* w_img,
                            float eps, const fa_rope_t* rope, const fa_tensor_t* dy,
                            const fa_tensor_t* dx_txt, const fa_tensor_t* dx_img, float* dw_txt,
                            float* dw_img, cudaStream_t stream) {
  const int S = T + I;
  const qkp::Seg txt = T > 0 ? make_seg(x_txt, w_txt) : make_seg(x_img, w_img);
  const qkp::Seg img = I > 0 ? make_seg(x_img, w_img) : txt;
  const fa_tensor_t* dxt = T > 0 ? dx_txt : dx_img;
  const fa_tensor_t* dxi = I > 0 ? dx_img : dx_txt;
  const RopeArgs r = make_rope_args(rope, 1, 0);
  const int tiles = (S + qkp::kTokens - 1) / qkp::kTokens;
  qkp::qk_norm_rope_bwd_kernel<<<(unsigned)((int64_t)B * tiles), qkp::kThreads, 0, stream>>>(
      txt, img, T, S, H, eps, r, qkp::View{dy->data, dy->stride_b, dy->stride_s, dy->stride_h},
      qkp::View{dxt->data, dxt->stride_b, dxt->stride_s, dxt->stride_h},
      qkp::View{dxi->data, dxi->stride_b, dxi->stride_s, dxi->stride_h},
      T > 0 ? dw_txt : nullptr, I > 0 ? dw_img : nullptr);
  return launch_status();
}

int qkp_device_status() { return tu_device_status(); }

}  // namespace fa
