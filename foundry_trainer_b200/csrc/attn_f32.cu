// attn_f32.cu — exact fp32 path of the joint-attention op (SIMT, no TF32).
//
// The reference runs its fp32 configuration with fp32 scores, softmax and
// matmuls (crates/foundry-spike/src/lib.rs:133-149 forward, :216-263
// backward); tensor cores cannot hold a 1e-4 max-relative bound in fp32
// (TF32 keeps 10 mantissa bits), so this path uses FFMA only:
//   fwd:   one CTA per 32 query rows, online softmax over 32-key tiles
//   dK/dV: one CTA per 32 keys, loops over 32-row query tiles
//   dQ:    one CTA per 32 query rows, loops over 32-key tiles
// No atomics: every output element has exactly one writer, so repeats are
// bit-identical.
#include "attn_common.h"
#include "sm100_ptx.cuh"

namespace fa {
namespace f32 {

constexpr int kT = 32;        // tile edge (rows and keys)
constexpr int kD = 128;
constexpr int kPad = kD + 1;  // padded row pitch for conflict-free column reads
constexpr int kThreads = 256;

struct View {
  const float* p;
  int64_t sb, ss, sh;
  __device__ __forceinline__ const float* row(int b, int s, int h) const {
    return p + (int64_t)b * sb + (int64_t)s * ss + (int64_t)h * sh;
  }
};
struct OutView {
  float* p;
  int64_t sb, ss, sh;
  __device__ __forceinline__ float* row(int b, int s, int h) const {
    return p + (int64_t)b * sb + (int64_t)s * ss + (int64_t)h * sh;
  }
};

// Loads rows [r0, r0+32) of a (S, D) slice into a padded shared tile; rows
// past `n` are zero.
__device__ __forceinline__ void load_tile(float* tile, const View& v, int b,
                                          int h, int r0, int n) {
  for (int idx = threadIdx.x; idx < kT * kD; idx += kThreads) {
    const int r = idx / kD, d = idx % kD;
    tile[r * kPad + d] = (r0 + r < n) ? v.row(b, r0 + r, h)[d] : 0.f;
  }
}

// ------------------------------------------------------------------ forward
__global__ void __launch_bounds__(kThreads)
fwd_kernel(View q, View k, View v, OutView o, float* lse, int S, int kv_len,
           int H, float scale) {
  extern __shared__ float sm[];
  float* sq = sm;                 // 32 x 129
  float* sk = sq + kT * kPad;     // 32 x 129
  float* sv = sk + kT * kPad;     // 32 x 129
  float* sp = sv + kT * kPad;     // 32 x 33
  const int q0 = blockIdx.x * kT, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x;
  const int r = t >> 3;       // query row of this thread
  const int g = t & 7;        // 8 threads per row
  load_tile(sq, q, b, h, q0, S);
  float m = -INFINITY, l = 0.f;
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  for (int k0 = 0; k0 < kv_len; k0 += kT) {
    __syncthreads();
    load_tile(sk, k, b, h, k0, kv_len);
    load_tile(sv, v, b, h, k0, kv_len);
    __syncthreads();
    float s[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = g * 4 + i;
      float a = 0.f;
      for (int d = 0; d < kD; ++d) a = fmaf(sq[r * kPad + d], sk[c * kPad + d], a);
      s[i] = (k0 + c < kv_len) ? a * scale : -INFINITY;
    }
    float mx = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m, mx);
    const float alpha = expf(m - m_new);
    float ps = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float e = expf(s[i] - m_new);
      sp[r * (kT + 1) + g * 4 + i] = e;
      ps += e;
    }
#pragma unroll
    for (int off = 1; off < 8; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    l = l * alpha + ps;
    m = m_new;
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int d = g * 16 + i;
      float a = acc[i] * alpha;
      for (int c = 0; c < kT; ++c) a = fmaf(sp[r * (kT + 1) + c], sv[c * kPad + d], a);
      acc[i] = a;
    }
  }
  const int row = q0 + r;
  if (row < S) {
    float* dst = o.row(b, row, h);
    const float inv = 1.f / l;
#pragma unroll
    for (int i = 0; i < 16; ++i) dst[g * 16 + i] = acc[i] * inv;
    if (g == 0) lse[((int64_t)b * H + h) * S + row] = m + logf(l);
  }
}

// ---------------------------------------------------------------- dK and dV
// For keys [k0, k0+32): dV = sum_q P^T dO, dK = scale * sum_q dS^T Q.
__global__ void __launch_bounds__(kThreads)
dkdv_kernel(View q, View k, View v, View d_o, const float* lse,
            const float* delta, OutView dk, OutView dv, int S, int H,
            float scale) {
  extern __shared__ float sm[];
  float* sk = sm;
  float* sv = sk + kT * kPad;
  float* sq = sv + kT * kPad;
  float* sd = sq + kT * kPad;
  float* sp = sd + kT * kPad;      // P^T: 32 keys x 33
  float* sds = sp + kT * (kT + 1); // dS^T
  float* slse = sds + kT * (kT + 1);
  float* sdel = slse + kT;
  const int k0 = blockIdx.x * kT, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, kr = t >> 3, g = t & 7;
  load_tile(sk, k, b, h, k0, S);
  load_tile(sv, v, b, h, k0, S);
  float adv[16], adk[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) adv[i] = adk[i] = 0.f;
  const float* lse_bh = lse + ((int64_t)b * H + h) * S;
  const float* del_bh = delta + ((int64_t)b * H + h) * S;
  for (int q0 = 0; q0 < S; q0 += kT) {
    __syncthreads();
    load_tile(sq, q, b, h, q0, S);
    load_tile(sd, d_o, b, h, q0, S);
    if (t < kT) {
      slse[t] = (q0 + t < S) ? lse_bh[q0 + t] : INFINITY;
      sdel[t] = (q0 + t < S) ? del_bh[q0 + t] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = g * 4 + i;  // query in tile
      float s = 0.f, dp = 0.f;
      for (int d = 0; d < kD; ++d) {
        s = fmaf(sk[kr * kPad + d], sq[c * kPad + d], s);
        dp = fmaf(sv[kr * kPad + d], sd[c * kPad + d], dp);
      }
      const float p = expf(s * scale - slse[c]);
      sp[kr * (kT + 1) + c] = p;
      sds[kr * (kT + 1) + c] = p * (dp - sdel[c]);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int d = g * 16 + i;
      float av = adv[i], ak = adk[i];
      for (int c = 0; c < kT; ++c) {
        av = fmaf(sp[kr * (kT + 1) + c], sd[c * kPad + d], av);
        ak = fmaf(sds[kr * (kT + 1) + c], sq[c * kPad + d], ak);
      }
      adv[i] = av;
      adk[i] = ak;
    }
  }
  const int key = k0 + kr;
  if (key < S) {
    float* pv = dv.row(b, key, h);
    float* pk = dk.row(b, key, h);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      pv[g * 16 + i] = adv[i];
      pk[g * 16 + i] = adk[i] * scale;
    }
  }
}

// ----------------------------------------------------------------------- dQ
__global__ void __launch_bounds__(kThreads)
dq_kernel(View q, View k, View v, View d_o, const float* lse,
          const float* delta, OutView dq, int S, int H, float scale) {
  extern __shared__ float sm[];
  float* sq = sm;
  float* sd = sq + kT * kPad;
  float* sk = sd + kT * kPad;
  float* sv = sk + kT * kPad;
  float* sds = sv + kT * kPad;  // dS: 32 queries x 33
  const int q0 = blockIdx.x * kT, h = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, r = t >> 3, g = t & 7;
  load_tile(sq, q, b, h, q0, S);
  load_tile(sd, d_o, b, h, q0, S);
  const int row = q0 + r;
  const float my_lse =
      (row < S) ? lse[((int64_t)b * H + h) * S + row] : INFINITY;
  const float my_del = (row < S) ? delta[((int64_t)b * H + h) * S + row] : 0.f;
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  for (int k0 = 0; k0 < S; k0 += kT) {
    __syncthreads();
    load_tile(sk, k, b, h, k0, S);
    load_tile(sv, v, b, h, k0, S);
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = g * 4 + i;
      float s = 0.f, dp = 0.f;
      for (int d = 0; d < kD; ++d) {
        s = fmaf(sq[r * kPad + d], sk[c * kPad + d], s);
        dp = fmaf(sd[r * kPad + d], sv[c * kPad + d], dp);
      }
      const float p = (k0 + c < S) ? expf(s * scale - my_lse) : 0.f;
      sds[r * (kT + 1) + c] = p * (dp - my_del);
    }
    __syncthreads();
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int d = g * 16 + i;
      float a = acc[i];
      for (int c = 0; c < kT; ++c) a = fmaf(sds[r * (kT + 1) + c], sk[c * kPad + d], a);
      acc[i] = a;
    }
  }
  if (row < S) {
    float* dst = dq.row(b, row, h);
#pragma unroll
    for (int i = 0; i < 16; ++i) dst[g * 16 + i] = acc[i] * scale;
  }
}

View view_of(const fa_tensor_t* t) {
  return View{reinterpret_cast<const float*>(t->data), t->stride_b, t->stride_s,
              t->stride_h};
}
OutView outview_of(const fa_tensor_t* t) {
  return OutView{reinterpret_cast<float*>(t->data), t->stride_b, t->stride_s,
                 t->stride_h};
}

}  // namespace f32

int launch_attn_fwd_f32(const AttnShape& sh, int kv_len, const fa_tensor_t* q,
                        const fa_tensor_t* k, const fa_tensor_t* v,
                        const fa_tensor_t* o, float* lse, float scale,
                        cudaStream_t stream) {
  const int smem = (3 * f32::kT * f32::kPad + f32::kT * (f32::kT + 1)) * 4;
  int rc = ensure_smem_attr((const void*)f32::fwd_kernel, smem, kKernelF32Fwd);
  if (rc) return rc;
  dim3 grid((sh.S + f32::kT - 1) / f32::kT, sh.H, sh.B);
  f32::fwd_kernel<<<grid, f32::kThreads, smem, stream>>>(
      f32::view_of(q), f32::view_of(k), f32::view_of(v), f32::outview_of(o),
      lse, sh.S, kv_len, sh.H, scale);
  return launch_status();
}

int launch_attn_bwd_f32(const AttnShape& sh, const fa_tensor_t* q,
                        const fa_tensor_t* k, const fa_tensor_t* v,
                        const fa_tensor_t* d_o, const float* lse,
                        const float* delta, const fa_tensor_t* dq,
                        const fa_tensor_t* dk, const fa_tensor_t* dv,
                        float scale, cudaStream_t stream) {
  const int smem_kv =
      (4 * f32::kT * f32::kPad + 2 * f32::kT * (f32::kT + 1) + 2 * f32::kT) * 4;
  const int smem_q = (4 * f32::kT * f32::kPad + f32::kT * (f32::kT + 1)) * 4;
  int rc = ensure_smem_attr((const void*)f32::dkdv_kernel, smem_kv, kKernelF32Bwd);
  if (rc) return rc;
  rc = ensure_smem_attr((const void*)f32::dq_kernel, smem_q, kKernelF32Bwd + 1);
  if (rc) return rc;
  dim3 grid((sh.S + f32::kT - 1) / f32::kT, sh.H, sh.B);
  f32::dkdv_kernel<<<grid, f32::kThreads, smem_kv, stream>>>(
      f32::view_of(q), f32::view_of(k), f32::view_of(v), f32::view_of(d_o),
      lse, delta, f32::outview_of(dk), f32::outview_of(dv), sh.S, sh.H, scale);
  if (launch_status() != FA_OK) return FA_ERR_LAUNCH;
  f32::dq_kernel<<<grid, f32::kThreads, smem_q, stream>>>(
      f32::view_of(q), f32::view_of(k), f32::view_of(v), f32::view_of(d_o),
      lse, delta, f32::outview_of(dq), sh.S, sh.H, scale);
  return launch_status();
}

int f32_device_status() { return tu_device_status(); }

}  // namespace fa
