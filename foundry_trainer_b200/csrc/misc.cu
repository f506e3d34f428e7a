// misc.cu — memory-bound helpers around the attention kernels:
//   * backward prologue: Delta = rowsum(dO * O) and the padded LSE*log2(e)
//     table the bf16 backward streams with each Q tile;
//   * axial RoPE apply / inverse (the reference's apply_rope, lib.rs:122-129);
//   * fp32 -> compute-dtype cast with scale and inverse rotation (dQ finish);
//   * log-sum-exp merge of two partial attention results (sequence shards).
// All are one pass over their rows; one warp per (b, s, h) row, lane l owns
// head-dim columns {l, l+32, l+64, l+96} so loads are coalesced and the
// rotate-half partner of column d (d +- 16 inside a 32-wide axis segment) is
// lane l ^ 16 holding the same slot.
#include <algorithm>

#include "attn_common.h"
#include "rope.cuh"
#include "sm100_ptx.cuh"

namespace fa {
namespace misc {

constexpr int kWarps = 8;

template <typename T>
__device__ __forceinline__ float ld_elem(const T* p);
template <>
__device__ __forceinline__ float ld_elem<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld_elem<__nv_bfloat16>(const __nv_bfloat16* p) {
  return __bfloat162float(*p);
}
template <typename T>
__device__ __forceinline__ void st_elem(T* p, float v);
template <>
__device__ __forceinline__ void st_elem<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st_elem<__nv_bfloat16>(__nv_bfloat16* p, float v) {
  *p = __float2bfloat16_rn(v);
}

struct TView {
  const void* p;
  int64_t sb, ss, sh;
};
struct TOut {
  void* p;
  int64_t sb, ss, sh;
};

// rows ordered (b, h, s) with s in [0, s_pad): writes delta (and lse2) rows
template <typename T>
__global__ void delta_kernel(TView o, TView d_o, const float* lse, float* delta,
                             float* lse2, int S, int H, int s_pad, int B) {
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * H * s_pad) return;
  const int s = (int)(row % s_pad);
  const int64_t bh = row / s_pad;
  const int h = (int)(bh % H), b = (int)(bh / H);
  float acc = 0.f;
  if (s < S) {
    const T* po = reinterpret_cast<const T*>(o.p) + b * o.sb + s * o.ss + h * o.sh;
    const T* pd = reinterpret_cast<const T*>(d_o.p) + b * d_o.sb + s * d_o.ss + h * d_o.sh;
#pragma unroll
    for (int a = 0; a < 4; ++a)
      acc = fmaf(ld_elem<T>(po + lane + 32 * a), ld_elem<T>(pd + lane + 32 * a), acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  if (lane == 0) {
    delta[row] = acc;
    if (lse2 != nullptr)
      lse2[row] = (s < S) ? lse[bh * S + s] * 1.4426950408889634f : INFINITY;
  }
}

// One warp per row: y = rot(x) (or the inverse), fp32 math, axis_dim == 32.
// blockIdx.y selects one of two (x, y) pairs so q and k rotate in one launch.
template <typename Tin, typename Tout>
__global__ void rope_warp_kernel(TView x0, TOut y0, TView x1, TOut y1, RopeArgs r,
                                 int S, int H, int B, float alpha, int inverse) {
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * S * H) return;
  const TView& x = blockIdx.y == 0 ? x0 : x1;
  const TOut& y = blockIdx.y == 0 ? y0 : y1;
  const int h = (int)(row % H);
  const int64_t bs = row / H;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const Tin* px = reinterpret_cast<const Tin*>(x.p) + b * x.sb + s * x.ss + h * x.sh;
  Tout* py = reinterpret_cast<Tout*>(y.p) + b * y.sb + s * y.ss + h * y.sh;
  float v[4];
#pragma unroll
  for (int a = 0; a < 4; ++a) v[a] = ld_elem<Tin>(px + lane + 32 * a) * alpha;
  if (r.pos != nullptr) {
    const int j = lane & 15;
    const bool first = lane < 16;
    // forward: y1 = x1 c - x2 s, y2 = x2 c + x1 s; inverse: the transpose
    const float sgn = (first != (inverse != 0)) ? -1.f : 1.f;
#pragma unroll
    for (int a = 0; a < 4; ++a) {
      const float other = __shfl_xor_sync(0xffffffffu, v[a], 16);
      if (a < r.n_axes) {
        const float2 cs = rope_cs(r, s, a * 16 + j);
        v[a] = __fadd_rn(__fmul_rn(v[a], cs.x), __fmul_rn(sgn * other, cs.y));
      }
    }
  }
#pragma unroll
  for (int a = 0; a < 4; ++a) st_elem<Tout>(py + lane + 32 * a, v[a]);
}

// (cos, sin) per (token, frequency), rounded to the compute dtype: evaluated
// once per call and reused by every head, batch and kernel of that call.
// __grid_constant__: inv_freq is indexed in parameter space, not copied to
// local memory per thread.
__global__ void rope_table_kernel(const __grid_constant__ RopeArgs r, int S, float2* table) {
  const int nf = r.n_axes * (r.axis_dim >> 1);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)S * nf) return;
  const int t = (int)(i / nf), f = (int)(i % nf);
  table[(int64_t)(t + r.pos_offset) * nf + f] = rope_cs_direct(r, t, f);
}

// The same table, and beside it the bf16 (cos, sin) pairs of the bf16 path
// packed in one 32-bit word per (token, frequency): cos in the low half, sin
// in the high half (exact: the values are already rounded to bf16). The
// forward kernel's in-tile rotation reads the packed form.
__global__ void rope_table2_kernel(const __grid_constant__ RopeArgs r, int S, float2* table,
                                   uint32_t* packed, uint32_t* clear, int64_t n_clear) {
  const int nf = r.n_axes * (r.axis_dim >> 1);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n_clear) clear[i] = 0u;
  if (i >= (int64_t)S * nf) return;
  const int t = (int)(i / nf), f = (int)(i % nf);
  const float2 cs = rope_cs_direct(r, t, f);
  const int64_t o = (int64_t)(t + r.pos_offset) * nf + f;
  table[o] = cs;
  // the packed row of a token with 64 frequencies is ordered for the forward
  // kernel's quarter-warp reads: words 4i..4i+3 hold frequencies 8i..8i+3,
  // words 32+4i..32+4i+3 hold 8i+4..8i+7
  const int fp = nf == 64 ? ((f >> 2) & 1) * 32 + (f >> 3) * 4 + (f & 3) : f;
  packed[o - f + fp] =
      (__float_as_uint(cs.x) >> 16) | (__float_as_uint(cs.y) & 0xFFFF0000u);
}

// ------------------------------------------------ token-major fast paths
// For the reference layout (head_dim 128 = four 32-wide axes) with a (cos,
// sin) table: one block per token, one warp per head row; lane l owns
// elements 4l..4l+3 (one 8- or 16-byte access per lane, a whole row per warp
// instruction); the rotate-half partner of element 4l+u is element 4(l^4)+u.
template <typename T>
struct Vec4;
template <>
struct Vec4<float> {
  static __device__ __forceinline__ void load(const float* p, float* v) {
    const float4 x = *reinterpret_cast<const float4*>(p);
    v[0] = x.x; v[1] = x.y; v[2] = x.z; v[3] = x.w;
  }
  static __device__ __forceinline__ void store(float* p, const float* v) {
    *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  }
};
template <>
struct Vec4<__nv_bfloat16> {
  static __device__ __forceinline__ void load(const __nv_bfloat16* p, float* v) {
    const uint2 x = *reinterpret_cast<const uint2*>(p);
    v[0] = __uint_as_float(x.x << 16); v[1] = __uint_as_float(x.x & 0xFFFF0000u);
    v[2] = __uint_as_float(x.y << 16); v[3] = __uint_as_float(x.y & 0xFFFF0000u);
  }
  static __device__ __forceinline__ void store(__nv_bfloat16* p, const float* v) {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
  }
};

// y = alpha * rot(x) (or the inverse rotation); blockIdx.x = token (b, s),
// blockIdx.y selects the (x, y) pair. Four warps; each first issues the loads
// of up to eight head rows, then the token's 64 (cos, sin) pairs are read
// from the table (or evaluated, without one) into shared memory while those
// loads are in flight, and the rows are rotated and stored.
constexpr int kRopeWarps = 4;
constexpr int kRopeRowsPerWarp = 8;
template <typename Tin, typename Tout>
__global__ void __launch_bounds__(32 * kRopeWarps)
rope_token_kernel(TView x0, TOut y0, TView x1, TOut y1,
                  const __grid_constant__ RopeArgs r, int S, int H, float alpha,
                  int inverse) {
  __shared__ float2 cs_s[64];
  const TView& x = blockIdx.y == 0 ? x0 : x1;
  const TOut& y = blockIdx.y == 0 ? y0 : y1;
  const int s = (int)(blockIdx.x % S), b = (int)(blockIdx.x / S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool rotate = r.pos != nullptr;
  const bool first = (lane & 7) < 4;  // element in the first half of its axis
  // forward: first half y = x c - x' s, second half y = x c + x' s;
  // inverse: the transposed rotation (signs swapped)
  const float sgn = (first != (inverse != 0)) ? -1.f : 1.f;
  const int f0 = (lane >> 3) * 16 + (lane & 3) * 4;  // lane's frequencies f0..f0+3
  float v[kRopeRowsPerWarp][4];
  auto load_rows = [&](int h0) {
#pragma unroll
    for (int k = 0; k < kRopeRowsPerWarp; ++k) {
      const int h = h0 + k * kRopeWarps;
      if (h < H)
        Vec4<Tin>::load(reinterpret_cast<const Tin*>(x.p) + b * x.sb + s * x.ss + h * x.sh + 4 * lane,
                        v[k]);
    }
  };
  load_rows(warp);
  float c[4], sn[4];
  if (rotate && threadIdx.x < 64) {
    const int64_t ti = (int64_t)(s + r.pos_offset) * 64 + threadIdx.x;
    const float2 t = r.table != nullptr ? r.table[ti] : rope_cs_direct(r, s, threadIdx.x);
    cs_s[threadIdx.x] = t;
    if (r.table_out != nullptr && b == 0 && blockIdx.y == 0) r.table_out[ti] = t;
  }
  __syncthreads();
  if (rotate) {
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      c[u] = cs_s[f0 + u].x;
      sn[u] = cs_s[f0 + u].y;
    }
  }
  for (int h0 = warp; h0 < H; h0 += kRopeRowsPerWarp * kRopeWarps) {
    if (h0 != warp) load_rows(h0);
#pragma unroll
    for (int k = 0; k < kRopeRowsPerWarp; ++k) {
      const int h = h0 + k * kRopeWarps;
      if (h >= H) break;  // uniform across the warp
#pragma unroll
      for (int u = 0; u < 4; ++u) v[k][u] *= alpha;
      if (rotate) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float other = __shfl_xor_sync(0xffffffffu, v[k][u], 4);
          v[k][u] = __fadd_rn(__fmul_rn(v[k][u], c[u]), __fmul_rn(sgn * other, sn[u]));
        }
      }
      Vec4<Tout>::store(reinterpret_cast<Tout*>(y.p) + b * y.sb + s * y.ss + h * y.sh + 4 * lane,
                        v[k]);
    }
  }
}

// dQ finish of the deterministic backward: y[b, s, h] = alpha *
// inverse_rope(x[0] + x[1] + ... + x[n_parts-1]) for the (b, h, s) row of
// the fp32 (n_parts, B, H, s_pad, 128) partials, summed left to right in
// slot order (so the same inputs give the same bits). One block per token
// (b, s); warp w handles heads w, w+4, ...; lane l owns elements 4l..4l+3
// and keeps eight slots' loads in flight.
__global__ void __launch_bounds__(32 * kRopeWarps)
dq_parts_finish_kernel(const float* x, int n_parts, int64_t part_stride, TOut y,
                       const __grid_constant__ RopeArgs r, int S, int H, int s_pad,
                       float alpha, int out_bf16) {
  __shared__ float2 cs_s[64];
  const int s = (int)(blockIdx.x % S), b = (int)(blockIdx.x / S);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bool rotate = r.pos != nullptr;
  if (rotate && threadIdx.x < 64) {
    const int64_t ti = (int64_t)(s + r.pos_offset) * 64 + threadIdx.x;
    cs_s[threadIdx.x] = r.table != nullptr ? r.table[ti] : rope_cs_direct(r, s, threadIdx.x);
  }
  __syncthreads();
  // inverse rotation: first half x c + x' s, second half x c - x' s
  const float sgn = (lane & 7) < 4 ? 1.f : -1.f;
  const int f0 = (lane >> 3) * 16 + (lane & 3) * 4;
  constexpr int kBatch = 8;
  for (int h = warp; h < H; h += kRopeWarps) {
    const float* src = x + (((int64_t)b * H + h) * s_pad + s) * 128 + 4 * lane;
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < n_parts; j0 += kBatch) {
      float4 t[kBatch];
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (j0 + u < n_parts)
          t[u] = __ldcs(reinterpret_cast<const float4*>(src + (int64_t)(j0 + u) * part_stride));
#pragma unroll
      for (int u = 0; u < kBatch; ++u)
        if (j0 + u < n_parts) {
          v[0] += t[u].x;
          v[1] += t[u].y;
          v[2] += t[u].z;
          v[3] += t[u].w;
        }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) v[u] *= alpha;
    if (rotate) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float other = __shfl_xor_sync(0xffffffffu, v[u], 4);
        const float2 cs = cs_s[f0 + u];
        v[u] = __fadd_rn(__fmul_rn(v[u], cs.x), __fmul_rn(sgn * other, cs.y));
      }
    }
    if (out_bf16)
      Vec4<__nv_bfloat16>::store(reinterpret_cast<__nv_bfloat16*>(y.p) + b * y.sb + s * y.ss +
                                     h * y.sh + 4 * lane, v);
    else
      Vec4<float>::store(reinterpret_cast<float*>(y.p) + b * y.sb + s * y.ss + h * y.sh + 4 * lane,
                         v);
  }
}

// bf16 -> bf16 rotation for the reference layout, eight tokens per block:
// lane l of a half-warp owns elements 8l..8l+7 of a row (one 16-byte access;
// the rotate-half partner of element 8l+u is element 8(l^2)+u), so a warp
// instruction moves two rows. All of a thread's row loads are issued before
// the block evaluates its tokens' (cos, sin) into shared memory.
constexpr int kTokTokens = 8;
constexpr int kTokThreads = 256;
constexpr int kTokMaxRows = 12;  // rows per thread: 8 tokens x H <= 16 x 12 = 192 (H <= 24)
__global__ void __launch_bounds__(kTokThreads)
rope_tok8_bf16_kernel(TView x0, TOut y0, TView x1, TOut y1,
                      const __grid_constant__ RopeArgs r, int S, int H, float alpha,
                      int inverse) {
  __shared__ float2 cs_s[kTokTokens][64];
  const TView& x = blockIdx.y == 0 ? x0 : x1;
  const TOut& y = blockIdx.y == 0 ? y0 : y1;
  const int tiles = (S + kTokTokens - 1) / kTokTokens;
  const int s0 = (int)(blockIdx.x % tiles) * kTokTokens, b = (int)(blockIdx.x / tiles);
  const int hw = threadIdx.x >> 4;  // half-warp: one row per access
  const int l = threadIdx.x & 15;
  const int rows = kTokTokens * H;
  const bool rotate = r.pos != nullptr;
  uint4 v[kTokMaxRows];
#pragma unroll
  for (int k = 0; k < kTokMaxRows; ++k) {
    const int row = hw + k * (kTokThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    if (row < rows && s < S)
      v[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x.p) +
                                              b * x.sb + (int64_t)s * x.ss + h * x.sh + 8 * l);
  }
  if (rotate) {
    for (int i = threadIdx.x; i < kTokTokens * 64; i += kTokThreads) {
      const int t = i >> 6, f = i & 63, s = s0 + t;
      if (s < S) {
        const int64_t ti = (int64_t)(s + r.pos_offset) * 64 + f;
        const float2 c = r.table != nullptr ? r.table[ti] : rope_cs_direct(r, s, f);
        cs_s[t][f] = c;
        if (r.table_out != nullptr && b == 0 && blockIdx.y == 0) r.table_out[ti] = c;
      }
    }
  }
  __syncthreads();
  // forward: first half y = x c - x' s, second half y = x c + x' s;
  // inverse: the transposed rotation (signs swapped)
  const bool first = (l & 3) < 2;
  const float sgn = (first != (inverse != 0)) ? -1.f : 1.f;
  const int f0 = (l >> 2) * 16 + (l & 1) * 8;  // frequencies f0..f0+7
#pragma unroll
  for (int k = 0; k < kTokMaxRows; ++k) {
    const int row = hw + k * (kTokThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    const bool live = row < rows && s < S;  // uniform per half-warp
    float e[8];
    e[0] = __uint_as_float(v[k].x << 16); e[1] = __uint_as_float(v[k].x & 0xFFFF0000u);
    e[2] = __uint_as_float(v[k].y << 16); e[3] = __uint_as_float(v[k].y & 0xFFFF0000u);
    e[4] = __uint_as_float(v[k].z << 16); e[5] = __uint_as_float(v[k].z & 0xFFFF0000u);
    e[6] = __uint_as_float(v[k].w << 16); e[7] = __uint_as_float(v[k].w & 0xFFFF0000u);
#pragma unroll
    for (int u = 0; u < 8; ++u) e[u] *= alpha;
    if (rotate) {
      // partner values from lane l^2 (all 32 lanes take part in the shuffle)
      float o[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) o[u] = __shfl_xor_sync(0xffffffffu, e[u], 2);
      if (live) {
        const int tt = t < kTokTokens ? t : 0;
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const float2 c = cs_s[tt][f0 + u];
          e[u] = __fadd_rn(__fmul_rn(e[u], c.x), __fmul_rn(sgn * o[u], c.y));
        }
      }
    }
    if (live)
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(y.p) + b * y.sb +
                                (int64_t)s * y.ss + h * y.sh + 8 * l) =
          make_uint4(pack_bf16(e[0], e[1]), pack_bf16(e[2], e[3]), pack_bf16(e[4], e[5]),
                     pack_bf16(e[6], e[7]));
  }
}

// delta / lse2 for bf16 O, dO with 16-byte accesses, eight tokens per block
// (rows (token, head), a half-warp per row, every load issued first); the
// block also clears its tokens' rows of the fp32 dQ accumulator
// (B, H, s_pad, 128) when zero_acc is given.
__global__ void __launch_bounds__(kTokThreads)
delta_tok8_bf16_kernel(TView o, TView d_o, const float* lse, float* delta, float* lse2,
                       float* zero_acc, int S, int H, int s_pad) {
  __shared__ float sums[kTokMaxRows * (kTokThreads / 16)];
  const int tiles = s_pad / kTokTokens;
  const int s0 = (int)(blockIdx.x % tiles) * kTokTokens, b = (int)(blockIdx.x / tiles);
  const int hw = threadIdx.x >> 4;
  const int l = threadIdx.x & 15;
  const int rows = kTokTokens * H;
  uint4 a[kTokMaxRows], g[kTokMaxRows];
#pragma unroll
  for (int k = 0; k < kTokMaxRows; ++k) {
    const int row = hw + k * (kTokThreads / 16);
    const int t = row / H, h = row - t * H, s = s0 + t;
    if (row < rows && s < S) {
      a[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(o.p) +
                                              b * o.sb + (int64_t)s * o.ss + h * o.sh + 8 * l);
      g[k] = *reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(d_o.p) +
                                              b * d_o.sb + (int64_t)s * d_o.ss + h * d_o.sh + 8 * l);
    } else {
      a[k] = make_uint4(0, 0, 0, 0);
      g[k] = make_uint4(0, 0, 0, 0);
    }
  }
  if (zero_acc != nullptr) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int i = threadIdx.x; i < rows * 32; i += kTokThreads) {
      const int row = i >> 5, c = i & 31;
      const int t = row / H, h = row - t * H;
      reinterpret_cast<float4*>(zero_acc + (((int64_t)b * H + h) * s_pad + s0 + t) * 128)[c] = z;
    }
  }
#pragma unroll
  for (int k = 0; k < kTokMaxRows; ++k) {
    const uint32_t av[4] = {a[k].x, a[k].y, a[k].z, a[k].w};
    const uint32_t gv[4] = {g[k].x, g[k].y, g[k].z, g[k].w};
    float acc = 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      acc = fmaf(__uint_as_float(av[u] << 16), __uint_as_float(gv[u] << 16), acc);
      acc = fmaf(__uint_as_float(av[u] & 0xFFFF0000u), __uint_as_float(gv[u] & 0xFFFF0000u), acc);
    }
#pragma unroll
    for (int off = 8; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    const int row = hw + k * (kTokThreads / 16);
    if (l == 0 && row < rows) sums[row] = acc;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < rows; i += kTokThreads) {
    const int h = i / kTokTokens, t = i % kTokTokens;
    const int64_t bh = (int64_t)b * H + h;
    const int s = s0 + t;
    delta[bh * s_pad + s] = sums[t * H + h];
    if (lse2 != nullptr)
      lse2[bh * s_pad + s] = (s < S) ? lse[bh * S + s] * 1.4426950408889634f : INFINITY;
  }
}

// delta[b, h, s] = sum_d dO * O over s < s_pad (0 past S); lse2 likewise
// (+inf past S). One block per 8 tokens of one b: each warp reduces rows
// (token, head) four at a time (a lane holds 4 elements of each), the sums
// meet in shared memory and every head's 8 results leave as one 32-byte
// store.
constexpr int kDeltaTokens = 8;
constexpr int kDeltaMaxHeads = 64;
template <typename T>
__global__ void __launch_bounds__(256)
delta_token_kernel(TView o, TView d_o, const float* lse, float* delta,
                   float* lse2, int S, int H, int s_pad) {
  __shared__ float sums[kDeltaMaxHeads][kDeltaTokens];
  const int tiles = s_pad / kDeltaTokens;
  const int s0 = (int)(blockIdx.x % tiles) * kDeltaTokens, b = (int)(blockIdx.x / tiles);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rows = kDeltaTokens * H;
  for (int r0 = warp * 4; r0 < rows; r0 += (blockDim.x >> 5) * 4) {
    float acc[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int r = r0 + u;
      const int t = r / H, h = r % H;
      const int s = s0 + t;
      acc[u] = 0.f;
      if (r < rows && s < S) {
        float a[4], g[4];
        Vec4<T>::load(reinterpret_cast<const T*>(o.p) + b * o.sb + s * o.ss + h * o.sh + 4 * lane, a);
        Vec4<T>::load(reinterpret_cast<const T*>(d_o.p) + b * d_o.sb + s * d_o.ss + h * d_o.sh + 4 * lane, g);
        acc[u] = a[0] * g[0] + a[1] * g[1] + a[2] * g[2] + a[3] * g[3];
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int u = 0; u < 4; ++u) acc[u] += __shfl_xor_sync(0xffffffffu, acc[u], off);
    if (lane < 4) {
      const int r = r0 + lane;
      float v = acc[0];
#pragma unroll
      for (int u = 1; u < 4; ++u) v = lane == u ? acc[u] : v;
      if (r < rows) sums[r % H][r / H] = v;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < H * kDeltaTokens; i += blockDim.x) {
    const int h = i / kDeltaTokens, t = i % kDeltaTokens;
    const int64_t bh = (int64_t)b * H + h;
    const int s = s0 + t;
    delta[bh * s_pad + s] = sums[h][t];
    if (lse2 != nullptr)
      lse2[bh * s_pad + s] = (s < S) ? lse[bh * S + s] * 1.4426950408889634f : INFINITY;
  }
}

// Generic thread-per-row rotation for other axis layouts.
template <typename Tin, typename Tout>
__global__ void rope_row_kernel(TView x, TOut y, RopeArgs r, int S, int H,
                                int B, float alpha, int inverse) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= (int64_t)B * S * H) return;
  const int h = (int)(row % H);
  const int64_t bs = row / H;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const Tin* px = reinterpret_cast<const Tin*>(x.p) + b * x.sb + s * x.ss + h * x.sh;
  Tout* py = reinterpret_cast<Tout*>(y.p) + b * y.sb + s * y.ss + h * y.sh;
  float v[128];
  for (int d = 0; d < 128; ++d) v[d] = ld_elem<Tin>(px + d) * alpha;
  if (r.pos != nullptr) rope_rotate_row128(r, s, v, inverse != 0);
  for (int d = 0; d < 128; ++d) st_elem<Tout>(py + d, v[d]);
}

// (o_acc, lse_acc) <- merge with (o_blk, lse_blk); rows (b, s, h).
template <typename T>
__global__ void lse_merge_kernel(float* o_acc, float* lse_acc, TView o_blk,
                                 const float* lse_blk, int S, int H, int B,
                                 int first) {
  const int64_t row = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= (int64_t)B * S * H) return;
  const int h = (int)(row % H);
  const int64_t bs = row / H;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const int64_t li = ((int64_t)b * H + h) * S + s;
  const T* pb = reinterpret_cast<const T*>(o_blk.p) + b * o_blk.sb + s * o_blk.ss + h * o_blk.sh;
  float* pa = o_acc + row * 128;
  const float lb = lse_blk[li];
  if (first) {
#pragma unroll
    for (int a = 0; a < 4; ++a) pa[lane + 32 * a] = ld_elem<T>(pb + lane + 32 * a);
    if (lane == 0) lse_acc[li] = lb;
    return;
  }
  const float la = lse_acc[li];
  const float mx = fmaxf(la, lb);
  const float wa = expf(la - mx), wb = expf(lb - mx);
  const float inv = 1.f / (wa + wb);
#pragma unroll
  for (int a = 0; a < 4; ++a) {
    const int d = lane + 32 * a;
    pa[d] = (pa[d] * wa + ld_elem<T>(pb + d) * wb) * inv;
  }
  __syncwarp();
  if (lane == 0) lse_acc[li] = mx + logf(wa + wb);
}

__global__ void add_f32_kernel(int64_t n4, float4* dst, const float4* src) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4;
       i += (int64_t)gridDim.x * blockDim.x) {
    float4 a = dst[i];
    const float4 b = src[i];
    a.x += b.x;
    a.y += b.y;
    a.z += b.z;
    a.w += b.w;
    dst[i] = a;
  }
}

__global__ void add_f32_tail_kernel(int64_t n, float* dst, const float* src) {
  const int64_t i = threadIdx.x;
  if (i < n) dst[i] += src[i];
}

TView tview(const fa_tensor_t* t) { return TView{t->data, t->stride_b, t->stride_s, t->stride_h}; }
TOut tout(const fa_tensor_t* t) { return TOut{t->data, t->stride_b, t->stride_s, t->stride_h}; }

}  // namespace misc

// 4-element vector accesses need rows aligned to 4 elements and strides that
// are multiples of 4 elements
template <typename V>
static bool aligned16(const V& t, int dtype) {
  const int64_t es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  return (reinterpret_cast<uintptr_t>(t.p) % (4 * es)) == 0 && t.sb % 4 == 0 &&
         t.ss % 4 == 0 && t.sh % 4 == 0;
}

// 16-byte accesses of 8 bf16: rows aligned to 8 elements, strides multiples of 8
template <typename V>
static bool aligned16_8(const V& t) {
  return (reinterpret_cast<uintptr_t>(t.p) % 16) == 0 && t.sb % 8 == 0 && t.ss % 8 == 0 &&
         t.sh % 8 == 0;
}

int launch_bwd_delta(int dtype, const AttnShape& sh, const fa_tensor_t* o,
                     const fa_tensor_t* d_o, const float* lse, float* delta,
                     float* lse2, int s_pad, cudaStream_t stream, float* zero_acc) {
  const misc::TView ov = misc::tview(o), dv = misc::tview(d_o);
  if (dtype == FA_DTYPE_BF16 && sh.D == 128 && sh.H <= 24 && s_pad % misc::kTokTokens == 0 &&
      aligned16_8(ov) && aligned16_8(dv)) {
    const dim3 grid((unsigned)((int64_t)sh.B * (s_pad / misc::kTokTokens)));
    misc::delta_tok8_bf16_kernel<<<grid, misc::kTokThreads, 0, stream>>>(
        ov, dv, lse, delta, lse2, zero_acc, sh.S, sh.H, s_pad);
    return launch_status();
  }
  if (zero_acc != nullptr) {
    const int rc = record_cuda_error(cudaMemsetAsync(
        zero_acc, 0, (size_t)sh.B * sh.H * s_pad * sh.D * sizeof(float), stream));
    if (rc != FA_OK) return rc;
  }
  if (sh.D == 128 && sh.H <= misc::kDeltaMaxHeads && s_pad % misc::kDeltaTokens == 0 &&
      aligned16(ov, dtype) && aligned16(dv, dtype)) {
    const dim3 grid((unsigned)((int64_t)sh.B * (s_pad / misc::kDeltaTokens)));
    if (dtype == FA_DTYPE_BF16)
      misc::delta_token_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(
          ov, dv, lse, delta, lse2, sh.S, sh.H, s_pad);
    else
      misc::delta_token_kernel<float><<<grid, 256, 0, stream>>>(
          ov, dv, lse, delta, lse2, sh.S, sh.H, s_pad);
    return launch_status();
  }
  const int64_t rows = (int64_t)sh.B * sh.H * s_pad;
  const dim3 grid((unsigned)((rows + misc::kWarps - 1) / misc::kWarps));
  if (dtype == FA_DTYPE_BF16)
    misc::delta_kernel<__nv_bfloat16><<<grid, 32 * misc::kWarps, 0, stream>>>(
        misc::tview(o), misc::tview(d_o), lse, delta, lse2, sh.S, sh.H, s_pad, sh.B);
  else
    misc::delta_kernel<float><<<grid, 32 * misc::kWarps, 0, stream>>>(
        misc::tview(o), misc::tview(d_o), lse, delta, lse2, sh.S, sh.H, s_pad, sh.B);
  return launch_status();
}

static int launch_rope_generic(int dtype_in, int dtype_out, const AttnShape& sh,
                               const misc::TView& x, const misc::TOut& y,
                               const RopeArgs& r, float alpha, int inverse,
                               cudaStream_t stream,
                               const misc::TView* xb = nullptr,
                               const misc::TOut* yb = nullptr) {
  const unsigned npairs = xb != nullptr ? 2u : 1u;
  const misc::TView x2 = xb != nullptr ? *xb : x;
  const misc::TOut y2 = yb != nullptr ? *yb : y;
  const int64_t rows = (int64_t)sh.B * sh.S * sh.H;
  const bool token_path =
      sh.D == 128 && (r.pos == nullptr || (r.axis_dim == 32 && r.n_axes == 4)) &&
      aligned16(x, dtype_in) && aligned16(y, dtype_out) && aligned16(x2, dtype_in) &&
      aligned16(y2, dtype_out);
  if (!token_path && r.table_out != nullptr) {
    // only the token-major kernel writes the table as it goes: build it here
    RopeArgs rt = r;
    rt.table = nullptr;
    const int64_t n = (int64_t)sh.S * rt.n_axes * (rt.axis_dim / 2);
    misc::rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(rt, sh.S, r.table_out);
    const int rc = launch_status();
    if (rc != FA_OK) return rc;
    RopeArgs rr = r;
    rr.table = r.table_out;
    rr.table_out = nullptr;
    return launch_rope_generic(dtype_in, dtype_out, sh, x, y, rr, alpha, inverse, stream, xb, yb);
  }
  if (token_path && dtype_in == FA_DTYPE_BF16 && dtype_out == FA_DTYPE_BF16 &&
      sh.H <= 24 && aligned16_8(x) && aligned16_8(y) && aligned16_8(x2) && aligned16_8(y2)) {
    const int tiles = (sh.S + misc::kTokTokens - 1) / misc::kTokTokens;
    const dim3 grid((unsigned)((int64_t)sh.B * tiles), npairs);
    misc::rope_tok8_bf16_kernel<<<grid, misc::kTokThreads, 0, stream>>>(x, y, x2, y2, r, sh.S,
                                                                       sh.H, alpha, inverse);
    return launch_status();
  }
  if (token_path) {
    const dim3 grid((unsigned)((int64_t)sh.B * sh.S), npairs);
#define FA_ROPE_T(TI, TO)                                                    \
  misc::rope_token_kernel<TI, TO><<<grid, 32 * misc::kRopeWarps, 0, stream>>>(x, y, x2, y2, r, sh.S, \
                                                           sh.H, alpha, inverse)
    if (dtype_in == FA_DTYPE_BF16 && dtype_out == FA_DTYPE_BF16) FA_ROPE_T(__nv_bfloat16, __nv_bfloat16);
    else if (dtype_in == FA_DTYPE_F32 && dtype_out == FA_DTYPE_BF16) FA_ROPE_T(float, __nv_bfloat16);
    else if (dtype_in == FA_DTYPE_F32 && dtype_out == FA_DTYPE_F32) FA_ROPE_T(float, float);
    else FA_ROPE_T(__nv_bfloat16, float);
#undef FA_ROPE_T
    return launch_status();
  }
  const bool warp_path = (r.pos == nullptr) || (r.axis_dim == 32 && r.n_axes <= 4);
  if (warp_path) {
    const dim3 grid((unsigned)((rows + misc::kWarps - 1) / misc::kWarps));
    const int nt = 32 * misc::kWarps;
#define FA_ROPE_W(TI, TO)                                                       \
  misc::rope_warp_kernel<TI, TO><<<dim3(grid.x, npairs), nt, 0, stream>>>(       \
      x, y, x2, y2, r, sh.S, sh.H, sh.B, alpha, inverse)
    if (dtype_in == FA_DTYPE_BF16 && dtype_out == FA_DTYPE_BF16) FA_ROPE_W(__nv_bfloat16, __nv_bfloat16);
    else if (dtype_in == FA_DTYPE_F32 && dtype_out == FA_DTYPE_BF16) FA_ROPE_W(float, __nv_bfloat16);
    else if (dtype_in == FA_DTYPE_F32 && dtype_out == FA_DTYPE_F32) FA_ROPE_W(float, float);
    else FA_ROPE_W(__nv_bfloat16, float);
#undef FA_ROPE_W
  } else {
    if (npairs == 2) {
      const int rc = launch_rope_generic(dtype_in, dtype_out, sh, x2, y2, r, alpha,
                                         inverse, stream);
      if (rc != FA_OK) return rc;
    }
    const dim3 grid((unsigned)((rows + 127) / 128));
#define FA_ROPE_R(TI, TO) \
  misc::rope_row_kernel<TI, TO><<<grid, 128, 0, stream>>>(x, y, r, sh.S, sh.H, sh.B, alpha, inverse)
    if (dtype_in == FA_DTYPE_BF16 && dtype_out == FA_DTYPE_BF16) FA_ROPE_R(__nv_bfloat16, __nv_bfloat16);
    else if (dtype_in == FA_DTYPE_F32 && dtype_out == FA_DTYPE_BF16) FA_ROPE_R(float, __nv_bfloat16);
    else if (dtype_in == FA_DTYPE_F32 && dtype_out == FA_DTYPE_F32) FA_ROPE_R(float, float);
    else FA_ROPE_R(__nv_bfloat16, float);
#undef FA_ROPE_R
  }
  return launch_status();
}

int launch_rope_table(int dtype, int S, const fa_rope_t* rope, int pos_offset,
                      float2* table, cudaStream_t stream) {
  const RopeArgs r = make_rope_args(rope, dtype == FA_DTYPE_BF16 ? 1 : 0, pos_offset);
  const int64_t n = (int64_t)S * r.n_axes * (r.axis_dim / 2);
  misc::rope_table_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(r, S, table);
  return launch_status();
}

int launch_rope_table2(int S, const fa_rope_t* rope, float2* table, uint32_t* packed,
                       uint32_t* clear, int64_t n_clear, cudaStream_t stream) {
  const RopeArgs r = make_rope_args(rope, 1, 0);
  const int64_t n = std::max<int64_t>((int64_t)S * r.n_axes * (r.axis_dim / 2), n_clear);
  misc::rope_table2_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(r, S, table, packed,
                                                                           clear, n_clear);
  return launch_status();
}

int launch_rope(int dtype, const AttnShape& sh, const fa_tensor_t* x,
                const fa_tensor_t* y, const fa_rope_t* rope, int inverse,
                int pos_offset, cudaStream_t stream, const float2* table) {
  RopeArgs r = make_rope_args(rope, dtype == FA_DTYPE_BF16 ? 1 : 0, pos_offset);
  r.table = table;
  return launch_rope_generic(dtype, dtype, sh, misc::tview(x), misc::tout(y), r,
                             1.f, inverse, stream);
}

int launch_rope_pair(int dtype, const AttnShape& sh, const fa_tensor_t* x0,
                     const fa_tensor_t* y0, const fa_tensor_t* x1,
                     const fa_tensor_t* y1, const fa_rope_t* rope, int inverse,
                     int pos_offset, cudaStream_t stream, const float2* table,
                     float2* table_out) {
  RopeArgs r = make_rope_args(rope, dtype == FA_DTYPE_BF16 ? 1 : 0, pos_offset);
  r.table = table;
  r.table_out = table_out;
  const misc::TView xb = misc::tview(x1);
  const misc::TOut yb = misc::tout(y1);
  return launch_rope_generic(dtype, dtype, sh, misc::tview(x0), misc::tout(y0), r,
                             1.f, inverse, stream, &xb, &yb);
}

int launch_cast_f32(int dtype, const AttnShape& sh, const float* x,
                    const fa_tensor_t* y, float alpha, const fa_rope_t* rope,
                    int pos_offset, cudaStream_t stream, const float2* table,
                    int s_pad) {
  RopeArgs r = make_rope_args(rope, dtype == FA_DTYPE_BF16 ? 1 : 0, pos_offset);
  r.table = table;
  const int64_t D = sh.D;
  // x is (B, S, H, D) contiguous, or (B, H, s_pad, D) when s_pad > 0
  const misc::TView xv =
      s_pad > 0 ? misc::TView{x, (int64_t)sh.H * s_pad * D, D, (int64_t)s_pad * D}
                : misc::TView{x, (int64_t)sh.S * sh.H * D, (int64_t)sh.H * D, D};
  return launch_rope_generic(FA_DTYPE_F32, dtype, sh, xv, misc::tout(y), r,
                             alpha, 1, stream);
}

int launch_dq_parts_finish(int dtype, const AttnShape& sh, const float* x, int n_parts,
                           int64_t part_stride, int s_pad, const fa_tensor_t* y, float alpha,
                           const fa_rope_t* rope, const float2* table, cudaStream_t stream) {
  if (sh.D != 128 || n_parts <= 0) return FA_ERR_UNSUPPORTED;
  if (rope != nullptr && (rope->axis_dim != 32 || rope->n_axes != 4)) return FA_ERR_UNSUPPORTED;
  const misc::TOut yo = misc::tout(y);
  const int es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  if (reinterpret_cast<uintptr_t>(yo.p) % (4 * es) != 0 || (yo.sb * es) % (4 * es) != 0 ||
      (yo.ss * es) % (4 * es) != 0 || (yo.sh * es) % (4 * es) != 0)
    return FA_ERR_ALIGNMENT;
  RopeArgs r = make_rope_args(rope, dtype == FA_DTYPE_BF16 ? 1 : 0, 0);
  r.table = table;
  const dim3 grid((unsigned)((int64_t)sh.B * sh.S));
  misc::dq_parts_finish_kernel<<<grid, 32 * misc::kRopeWarps, 0, stream>>>(
      x, n_parts, part_stride, yo, r, sh.S, sh.H, s_pad, alpha, dtype == FA_DTYPE_BF16);
  return launch_status();
}

int launch_add_f32(int64_t n, float* dst, const float* src, cudaStream_t stream) {
  const int64_t n4 = n / 4;
  if (n4 > 0) {
    // 148 SMs x 8 blocks of 256 threads, grid-stride over float4
    const int64_t blocks = std::min<int64_t>((n4 + 255) / 256, 148 * 8);
    misc::add_f32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(
        n4, reinterpret_cast<float4*>(dst), reinterpret_cast<const float4*>(src));
  }
  if (n % 4 != 0)
    misc::add_f32_tail_kernel<<<1, 32, 0, stream>>>(n % 4, dst + 4 * n4, src + 4 * n4);
  return launch_status();
}

int launch_lse_merge(int dtype, const AttnShape& sh, float* o_acc,
                     float* lse_acc, const fa_tensor_t* o_blk,
                     const float* lse_blk, int first, cudaStream_t stream) {
  const int64_t rows = (int64_t)sh.B * sh.S * sh.H;
  const dim3 grid((unsigned)((rows + misc::kWarps - 1) / misc::kWarps));
  if (dtype == FA_DTYPE_BF16)
    misc::lse_merge_kernel<__nv_bfloat16><<<grid, 32 * misc::kWarps, 0, stream>>>(
        o_acc, lse_acc, misc::tview(o_blk), lse_blk, sh.S, sh.H, sh.B, first);
  else
    misc::lse_merge_kernel<float><<<grid, 32 * misc::kWarps, 0, stream>>>(
        o_acc, lse_acc, misc::tview(o_blk), lse_blk, sh.S, sh.H, sh.B, first);
  return launch_status();
}

int misc_device_status() { return tu_device_status(); }

}  // namespace fa
