// peer.cu — the device side of the sequence-parallel exchange between the
// GPUs of one node (one process per GPU).
//
// The reference runs its attention op on one device; at 512 + 128x128 tokens
// the sequence is sharded over the GPUs and every rank needs every K/V shard
// (forward) and every owner needs the dK/dV contributions of every rank's
// query rows (backward). On B200 the GPUs of a node share NVLink 5 through
// NVSwitch, so the exchange is done with the hardware directly:
//   * buffers that peers read or write are plain device allocations shared
//     through CUDA IPC handles (no multicast object is created);
//   * K/V shards are pulled from a peer's buffer by the copy engines
//     (cudaMemcpy2DAsync) or by a copy kernel whose small CTAs fit beside the
//     attention CTAs; either runs under the attention kernels;
//   * the backward kernel's epilogue stores each dK/dV row straight into the
//     owner rank's receive slot (attn_bwd_sm100.cu, scatter mode);
//   * ranks order these steps with a small barrier kernel over flags in the
//     peers' memory: release stores at system scope, acquire loads, and a
//     wait bounded in wall time that reports FA_ERR_DEVICE_TIMEOUT.
// This file also holds the two reductions of that path: the sum of the W
// dK/dV contributions an owner receives (with the inverse RoPE and the cast
// to bf16) and the merge of two fp32 (O, LSE) partial accumulators.
#include <algorithm>

#include "attn_common.h"
#include "rope.cuh"
#include "sm100_ptx.cuh"

namespace fa {
namespace peer {

// Flag block of one rank: arrive[channel][source rank], then the per-channel
// epoch this rank last completed (read and advanced by the barrier kernel, so
// the kernel can be captured in a CUDA graph).
constexpr int kArriveWords = FA_PEER_CHANNELS * FA_PEER_MAX;

// Output rows: element strides of a (B, S, H, D) tensor, unit stride in D.
struct OutView {
  void* p;
  int64_t sb, ss, sh;
};

struct BarrierArgs {
  uint32_t* flags[FA_PEER_MAX];
  int rank, world, channel;
  unsigned long long timeout_ns;
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// One warp. Lane p (p != rank) tells rank p that this rank has reached
// epoch e on the channel, then waits until rank p has told it the same. Every
// write this device made before the barrier (this and earlier kernels on the
// stream, peer stores included) is ordered before the flag by the
// system-scope fence and release store.
__global__ void __launch_bounds__(32) peer_barrier_kernel(const __grid_constant__ BarrierArgs a) {
  const int p = threadIdx.x;
  uint32_t* mine = a.flags[a.rank];
  uint32_t* epoch = mine + kArriveWords + a.channel;
  const uint32_t e = *reinterpret_cast<volatile uint32_t*>(epoch) + 1u;
  const bool peer = p < a.world && p != a.rank;
  if (peer) {
    __threadfence_system();
    st_release_sys(a.flags[p] + a.channel * FA_PEER_MAX + a.rank, e);
  }
  bool ok = true;
  if (peer) {
    const uint32_t* f = mine + a.channel * FA_PEER_MAX + p;
    const unsigned long long t0 = global_ns();
    while ((int)(ld_acquire_sys(f) - e) < 0) {
      if (global_ns() - t0 > a.timeout_ns) {
        ok = false;
        break;
      }
      __nanosleep(100);
    }
  }
  if (!ok) report_status(FA_ERR_DEVICE_TIMEOUT);
  __syncwarp();
  if (p == 0) *reinterpret_cast<volatile uint32_t*>(epoch) = e;
}

// y = alpha * inverse_rope(sum_p x[p]) as bf16/fp32 rows (blockIdx.y == 0),
// and y2 = sum_p x2[p] (blockIdx.y == 1, no rotation); x, x2 contiguous fp32
// (B, S, H, D) with parts `part_stride` floats apart. One warp per (b, s, h)
// row, lane l owns elements 4l..4l+3 (partner of 4l+u under rotate-half:
// lane l^4), all part loads issued before the sum.
constexpr int kRowsPerBlock = 8;
template <typename Tout>
__global__ void __launch_bounds__(32 * kRowsPerBlock)
reduce_cast_kernel(const float* x, const float* x2, int n_parts, int64_t part_stride,
                   OutView y, OutView y2, float alpha, const __grid_constant__ RopeArgs r,
                   int S, int H, int64_t rows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowsPerBlock + warp;
  if (row >= rows) return;
  const bool second = blockIdx.y == 1;
  const float* src = (second ? x2 : x) + row * 128 + 4 * lane;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kBatch = 8;
  for (int p0 = 0; p0 < n_parts; p0 += kBatch) {
    float4 t[kBatch];
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (p0 + u < n_parts)
        t[u] = __ldcs(reinterpret_cast<const float4*>(src + (int64_t)(p0 + u) * part_stride));
#pragma unroll
    for (int u = 0; u < kBatch; ++u)
      if (p0 + u < n_parts) {
        acc.x += t[u].x;
        acc.y += t[u].y;
        acc.z += t[u].z;
        acc.w += t[u].w;
      }
  }
  float v[4] = {acc.x * (second ? 1.f : alpha), acc.y * (second ? 1.f : alpha),
                acc.z * (second ? 1.f : alpha), acc.w * (second ? 1.f : alpha)};
  const int h = (int)(row % H);
  const int64_t bs = row / H;
  const int s = (int)(bs % S), b = (int)(bs / S);
  if (!second && r.pos != nullptr) {
    // inverse rotation: first half x c + x' s, second half x c - x' s
    const bool first = (lane & 7) < 4;
    const float sgn = first ? 1.f : -1.f;
    const int f0 = (lane >> 3) * 16 + (lane & 3) * 4;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float2 cs = rope_cs(r, s, f0 + u);
      const float other = __shfl_xor_sync(0xffffffffu, v[u], 4);
      v[u] = __fadd_rn(__fmul_rn(v[u], cs.x), __fmul_rn(sgn * other, cs.y));
    }
  }
  const OutView& o = second ? y2 : y;
  Tout* dst = reinterpret_cast<Tout*>(o.p) + b * o.sb + s * o.ss + h * o.sh + 4 * lane;
  if constexpr (sizeof(Tout) == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// Merge of two partial results over disjoint key sets, each an fp32 O
// (normalised rows, (B, S, H, D)) with its natural-log LSE ((B, H, S)):
//   LSE = log(e^a + e^b),  O = (e^a O_a + e^b O_b) / (e^a + e^b)
// One warp per row; lane l owns elements 4l..4l+3.
template <typename Tout>
__global__ void __launch_bounds__(32 * kRowsPerBlock)
merge2_kernel(const float* o_a, const float* lse_a, const float* o_b, const float* lse_b,
              OutView o, float* lse, int S, int H, int64_t rows) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowsPerBlock + warp;
  if (row >= rows) return;
  const int h = (int)(row % H);
  const int64_t bs = row / H;
  const int s = (int)(bs % S), b = (int)(bs / S);
  const int64_t li = ((int64_t)b * H + h) * S + s;
  const float4 xa = __ldcs(reinterpret_cast<const float4*>(o_a + row * 128) + lane);
  const float4 xb = __ldcs(reinterpret_cast<const float4*>(o_b + row * 128) + lane);
  const float la = lse_a[li], lb = lse_b[li];
  const float mx = fmaxf(la, lb);
  const float ea = expf(la - mx), eb = expf(lb - mx);
  const float inv = 1.f / (ea + eb);
  const float wa = ea * inv, wb = eb * inv;
  const float v[4] = {fmaf(xa.x, wa, xb.x * wb), fmaf(xa.y, wa, xb.y * wb),
                      fmaf(xa.z, wa, xb.z * wb), fmaf(xa.w, wa, xb.w * wb)};
  Tout* dst = reinterpret_cast<Tout*>(o.p) + b * o.sb + s * o.ss + h * o.sh + 4 * lane;
  if constexpr (sizeof(Tout) == 2) {
    *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16(v[0], v[1]), pack_bf16(v[2], v[3]));
  } else {
    *reinterpret_cast<float4*>(dst) = make_float4(v[0], v[1], v[2], v[3]);
  }
  if (lane == 0) lse[li] = mx + logf(ea + eb);
}

// One row (blockIdx.y) of width 16-byte units per grid row, copied by SMs
// with 16-byte loads and stores, 4 in flight per thread. Four warps, at most
// 40 registers and no shared memory: a CTA fits beside one attention CTA on
// an SM (which leaves ~6400 registers and ~1.8 KB of shared memory), so the
// copy runs under the forward's folds. Sources may be peers' memory.
constexpr int kCopyThreads = 128;
constexpr int kCopyUnroll = 4;
__global__ void __launch_bounds__(kCopyThreads, 12)
copy_rows_kernel(uint8_t* dst, int64_t dpitch, const uint8_t* src, int64_t spitch, int64_t w16) {
  const uint4* s = reinterpret_cast<const uint4*>(src + (int64_t)blockIdx.y * spitch);
  uint4* d = reinterpret_cast<uint4*>(dst + (int64_t)blockIdx.y * dpitch);
  const int64_t stride = (int64_t)gridDim.x * kCopyThreads;
  int64_t i = (int64_t)blockIdx.x * kCopyThreads + threadIdx.x;
  for (; i + (kCopyUnroll - 1) * stride < w16; i += kCopyUnroll * stride) {
    uint4 v[kCopyUnroll];
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) v[u] = __ldcs(s + i + u * stride);
#pragma unroll
    for (int u = 0; u < kCopyUnroll; ++u) d[i + u * stride] = v[u];
  }
  for (; i < w16; i += stride) d[i] = __ldcs(s + i);
}

}  // namespace peer

int launch_copy2d_sm(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                     size_t height, int ctas, cudaStream_t stream) {
  const int64_t w16 = (int64_t)(width / 16);
  const int per_row = std::max(1, ctas / (int)std::min<size_t>(height, (size_t)ctas));
  peer::copy_rows_kernel<<<dim3(per_row, (unsigned)height), peer::kCopyThreads, 0, stream>>>(
      reinterpret_cast<uint8_t*>(dst), (int64_t)dpitch, reinterpret_cast<const uint8_t*>(src),
      (int64_t)spitch, w16);
  return launch_status();
}

int launch_peer_barrier(int rank, int world, void* const* flags, int channel,
                        double timeout_s, cudaStream_t stream) {
  peer::BarrierArgs a{};
  for (int i = 0; i < world; ++i) a.flags[i] = reinterpret_cast<uint32_t*>(flags[i]);
  a.rank = rank;
  a.world = world;
  a.channel = channel;
  a.timeout_ns = (unsigned long long)(timeout_s * 1e9);
  peer::peer_barrier_kernel<<<1, 32, 0, stream>>>(a);
  return launch_status();
}

int launch_reduce_cast(int dtype, const AttnShape& sh, const float* x, const float* x2,
                       int n_parts, int64_t part_stride, const fa_tensor_t* y,
                       const fa_tensor_t* y2, float alpha, const fa_rope_t* rope,
                       cudaStream_t stream) {
  RopeArgs r = make_rope_args(rope, dtype == FA_DTYPE_BF16 ? 1 : 0, 0);
  const int64_t rows = (int64_t)sh.B * sh.S * sh.H;
  const peer::OutView o1{y->data, y->stride_b, y->stride_s, y->stride_h};
  const peer::OutView o2 = y2 ? peer::OutView{y2->data, y2->stride_b, y2->stride_s, y2->stride_h} : o1;
  const dim3 grid((unsigned)((rows + peer::kRowsPerBlock - 1) / peer::kRowsPerBlock),
                  y2 ? 2u : 1u);
  if (dtype == FA_DTYPE_BF16)
    peer::reduce_cast_kernel<__nv_bfloat16><<<grid, 32 * peer::kRowsPerBlock, 0, stream>>>(
        x, x2, n_parts, part_stride, o1, o2, alpha, r, sh.S, sh.H, rows);
  else
    peer::reduce_cast_kernel<float><<<grid, 32 * peer::kRowsPerBlock, 0, stream>>>(
        x, x2, n_parts, part_stride, o1, o2, alpha, r, sh.S, sh.H, rows);
  return launch_status();
}

int launch_merge2(int dtype, const AttnShape& sh, const float* o_a, const float* lse_a,
                  const float* o_b, const float* lse_b, const fa_tensor_t* o, float* lse,
                  cudaStream_t stream) {
  const int64_t rows = (int64_t)sh.B * sh.S * sh.H;
  const peer::OutView oo{o->data, o->stride_b, o->stride_s, o->stride_h};
  const dim3 grid((unsigned)((rows + peer::kRowsPerBlock - 1) / peer::kRowsPerBlock));
  if (dtype == FA_DTYPE_BF16)
    peer::merge2_kernel<__nv_bfloat16><<<grid, 32 * peer::kRowsPerBlock, 0, stream>>>(
        o_a, lse_a, o_b, lse_b, oo, lse, sh.S, sh.H, rows);
  else
    peer::merge2_kernel<float><<<grid, 32 * peer::kRowsPerBlock, 0, stream>>>(
        o_a, lse_a, o_b, lse_b, oo, lse, sh.S, sh.H, rows);
  return launch_status();
}

int peer_device_status() { return tu_device_status(); }

}  // namespace fa
