// attn_fwd_sm100.cu — bf16 joint-attention forward for sm_100a.
//
// Computes, per (batch, head), O = softmax(Q K^T * scale) V and the fp32
// log-sum-exp of each row: the forward of the reference op
// (crates/foundry-spike/src/lib.rs:133-149: fp32 scores, fp32 softmax, P in
// the compute dtype, PV with fp32 accumulation). Rounding difference: the
// reference rounds the normalised probabilities to bf16; this kernel rounds
// the unnormalised exp tile to bf16 and divides by the fp32 row sum at the
// end (both are one bf16 rounding of P; the LSE itself is fp32).
//
// One CTA owns one 128-row Q tile of one (b, h) and streams 128-key K/V
// tiles through TMA rings (K: 2 stages, V: 3 stages), starting at K/V tile
// `q_tile` and wrapping, so the CTAs of one head do not all request the same
// tile from L2 at once (the online softmax is order-independent):
//   warp 8      TMA producer of Q and K (one lane)
//   warp 10     TMA producer of V (one lane), so each ring fills as soon as
//               its own stage frees
//   warp 9      tcgen05 MMA issuer (one lane), TMEM owner
//   warps 0-7   softmax, O rescale and epilogue: two warpgroups, each thread
//               owns half a Q row (warpgroup 0 keys/columns 0-63, warpgroup 1
//               64-127); the row maximum is combined through shared memory.
// TMEM (512 columns): S_a [0,128) S_b [128,256) P_a [256,320) P_b [320,384)
// O [384,512). S and P are double-buffered: S(j+1) = Q K_{j+1}^T runs on the
// tensor core while the softmax of tile j runs, and the softmax of tile j+1
// writes its P (bf16, two per column; the TMEM A operand of O += P V) while
// PV(j) still reads the other buffer. No MMA waits for another to drain.
#include "attn_common.h"
#include "sm100_ptx.cuh"

namespace fa {
namespace fwd {

constexpr int kRows = 128;          // Q rows per CTA
constexpr int kKeys = 128;          // keys per K/V tile
constexpr int kTileBytes = 32768;   // 128 x 128 bf16
constexpr int kBlkBytes = 16384;    // one 64-column swizzle block
constexpr int kKStages = 2;
constexpr int kVStages = 3;
constexpr int kThreads = 352;

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kOffQ = 0;
constexpr int kOffK = kOffQ + kTileBytes;
constexpr int kOffV = kOffK + kKStages * kTileBytes;
constexpr int kOffBar = kOffV + kVStages * kTileBytes;
constexpr int kNumBars = 20;
// [3][2][128] fp32: row maxima of the two halves for even / odd KV tiles, then
// the two halves' row sums for the epilogue
constexpr int kOffRed = kOffBar + kNumBars * 8;
constexpr int kOffMisc = kOffRed + 3 * 2 * 128 * 4;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack

// barrier indices
constexpr int B_Q = 0;
constexpr int B_KFULL = 1;    // + stage (2)
constexpr int B_KEMPTY = 3;   // + stage (2)
constexpr int B_VFULL = 5;    // + stage (3)
constexpr int B_VEMPTY = 8;   // + stage (3)
constexpr int B_SFULL = 11;   // + S buffer (2)
constexpr int B_PREADY = 13;  // + P buffer (2): softmax wrote P(j), read S(j)
constexpr int B_PVDONE = 15;  // + P buffer (2): O += P(j) V_j completed
constexpr int B_FINAL = 17;

constexpr uint32_t kColS = 0;
constexpr uint32_t kColP = 256;  // + 64 * (j & 1)
constexpr uint32_t kColO = 384;

// K/V tile visited at step j by the CTA of Q tile `q_tile`.
__device__ __forceinline__ int kv_tile_of(int j, int q_tile, int nkv) {
  const int t = j + q_tile % nkv;
  return t >= nkv ? t - nkv : t;
}

struct Params {
  int S, H, kv_len, nkv;
  float scale_log2;  // scale * log2(e)
  __nv_bfloat16* o;
  int64_t os_b, os_s, os_h;
  float* lse;  // (B, H, S)
};

__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + kOffMisc + 4);

  const int warp = warp_id();
  const int lane = lane_id();
  const int q_tile = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int nkv = p.nkv;

  if (threadIdx.x == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int s = 0; s < kKStages; ++s) {
      mbar_init(&bars[B_KFULL + s], 1);
      mbar_init(&bars[B_KEMPTY + s], 1);
    }
    for (int s = 0; s < kVStages; ++s) {
      mbar_init(&bars[B_VFULL + s], 1);
      mbar_init(&bars[B_VEMPTY + s], 1);
    }
    mbar_init(&bars[B_SFULL + 0], 1);
    mbar_init(&bars[B_SFULL + 1], 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bars[B_PREADY + t], 256);
      mbar_init(&bars[B_PVDONE + t], 1);
    }
    mbar_init(&bars[B_FINAL], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // --------------------------------------------------- producer: Q and K
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      const int row = q_tile * kRows;
      mbar_arrive_expect_tx(&bars[B_Q], kTileBytes);
      tma_load_4d(smem + kOffQ, &tm_q, &bars[B_Q], 0, row, h, b);
      tma_load_4d(smem + kOffQ + kBlkBytes, &tm_q, &bars[B_Q], 64, row, h, b);
      bool ok = true;
      for (int jk = 0; jk < nkv; ++jk) {
        if (*abort_flag) break;
        const int s = jk % kKStages, n = jk / kKStages;
        if (jk >= kKStages && !(ok = mbar_wait(&bars[B_KEMPTY + s], (n - 1) & 1))) break;
        uint8_t* d = smem + kOffK + s * kTileBytes;
        mbar_arrive_expect_tx(&bars[B_KFULL + s], kTileBytes);
        const int krow = kv_tile_of(jk, q_tile, nkv) * kKeys;
        tma_load_4d(d, &tm_k, &bars[B_KFULL + s], 0, krow, h, b);
        tma_load_4d(d + kBlkBytes, &tm_k, &bars[B_KFULL + s], 64, krow, h, b);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 10) {
    // ------------------------------------------------------- producer: V
    if (lane == 0) {
      tma_prefetch_desc(&tm_v);
      bool ok = true;
      for (int jv = 0; jv < nkv; ++jv) {
        if (*abort_flag) break;
        const int s = jv % kVStages, n = jv / kVStages;
        if (jv >= kVStages && !(ok = mbar_wait(&bars[B_VEMPTY + s], (n - 1) & 1))) break;
        uint8_t* d = smem + kOffV + s * kTileBytes;
        mbar_arrive_expect_tx(&bars[B_VFULL + s], kTileBytes);
        const int vrow = kv_tile_of(jv, q_tile, nkv) * kKeys;
        tma_load_4d(d, &tm_v, &bars[B_VFULL + s], 0, vrow, h, b);
        tma_load_4d(d + kBlkBytes, &tm_v, &bars[B_VFULL + s], 64, vrow, h, b);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 9) {
    // ----------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t kIdescO = idesc_bf16(128, 128, false, true);
      const uint32_t q_base = smem_u32(smem + kOffQ);
      bool ok = mbar_wait(&bars[B_Q], 0);
      tc_fence_after();
      // S(j) = Q K_j^T into S buffer j&1
      auto issue_s = [&](int j) -> bool {
        const int s = j % kKStages, n = j / kKStages;
        if (!mbar_wait(&bars[B_KFULL + s], n & 1)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(smem + kOffK + s * kTileBytes);
        const uint32_t d = tmem + kColS + (uint32_t)(j & 1) * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss(d, kmajor_desc(q_base, kk, kBlkBytes),
                  kmajor_desc(k_base, kk, kBlkBytes), kIdescS, kk > 0);
        umma_commit(&bars[B_SFULL + (j & 1)]);
        umma_commit(&bars[B_KEMPTY + s]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkv > 1) ok = issue_s(1);
      for (int j = 0; ok && j < nkv; ++j) {
        if (*abort_flag) { ok = false; break; }
        const int s = j % kVStages, n = j / kVStages;
        if (!(ok = mbar_wait(&bars[B_VFULL + s], n & 1))) break;
        if (!(ok = mbar_wait(&bars[B_PREADY + (j & 1)], (j >> 1) & 1))) break;
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + kOffV + s * kTileBytes);
        const uint32_t p_col = kColP + (uint32_t)(j & 1) * 64u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts(tmem + kColO, tmem + p_col + kk * 8,
                  mnmajor_desc(v_base, kk, kBlkBytes), kIdescO,
                  (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&bars[B_PVDONE + (j & 1)]);
        umma_commit(&bars[B_VEMPTY + s]);
        // S buffer j&1 was read by softmax(j) before it signalled P ready.
        if (j + 2 < nkv) ok = issue_s(j + 2);
      }
      if (!ok) *abort_flag = 1;
      // drain: every MMA issued above completes before TMEM is released
      umma_commit(&bars[B_FINAL]);
      mbar_wait(&bars[B_FINAL], 0);
    }
  } else {
    // ----------------------------------------------- softmax warpgroups
    const int wg = warp >> 2;                 // column half of the row
    const int sub = warp & 3;                 // TMEM lane quarter
    const int row_in_tile = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t t_p0 = tmem + lane_off + kColP + (uint32_t)wg * 32u;
    const uint32_t t_o = tmem + lane_off + kColO + (uint32_t)wg * 64u;
    float* red = reinterpret_cast<float*>(smem + kOffRed);  // [j&1][wg][row]
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;  // this half's share of the row sum
    bool failed = false;
    for (int j = 0; j < nkv; ++j) {
      bool stop = failed || *abort_flag != 0;
      if (!stop) stop = !mbar_wait(&bars[B_SFULL + (j & 1)], (j >> 1) & 1);
      stop = __any_sync(0xffffffffu, stop);
      uint32_t sr[64];
      float mx = -INFINITY;
      if (!stop) {
        tc_fence_after();
        const uint32_t t_s =
            tmem + lane_off + kColS + (uint32_t)(j & 1) * 128u + (uint32_t)wg * 64u;
        tmem_ld32(t_s + 0, sr);
        tmem_ld32(t_s + 32, sr + 32);
        tmem_wait_ld();
        float* sv = reinterpret_cast<float*>(sr);
        const int valid = p.kv_len - kv_tile_of(j, q_tile, nkv) * kKeys - wg * 64;
        if (valid < 64) {
#pragma unroll
          for (int c = 0; c < 64; ++c)
            if (c >= valid) sv[c] = -INFINITY;
        }
        // pairwise tree: 6 dependent steps instead of a 63-long chain
        float m32[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) m32[c] = fmaxf(sv[c], sv[c + 32]);
#pragma unroll
        for (int w = 16; w >= 1; w >>= 1)
#pragma unroll
          for (int c = 0; c < w; ++c) m32[c] = fmaxf(m32[c], m32[c + w]);
        mx = m32[0];
        red[((j & 1) * 2 + wg) * 128 + row_in_tile] = mx;
      }
      // both halves leave together; after this the partner's maximum is visible
      if (named_bar_any(1, 256, stop)) break;
      mx = fmaxf(mx, red[((j & 1) * 2 + (wg ^ 1)) * 128 + row_in_tile]);
      float* sv = reinterpret_cast<float*>(sr);
      const float m_cand = mx * sl2;
      float m_use = m_run;
      float alpha = 1.f;
      // Keep the running maximum unless it grew by more than 2^8: P stays
      // <= 256 (exact range in bf16 and fp32) and O is rescaled only when
      // the maximum really moves; the result is the same up to rounding.
      if (m_cand > m_run + 8.f) {
        m_use = m_cand;
        alpha = fast_exp2(m_run - m_cand);  // 0 when m_run == -inf
      }
      // exponentials: every fourth on the FMA pipe (polynomial), the rest on
      // MUFU; four partial sums keep the additions off one dependent chain
      float sum4[4] = {0.f, 0.f, 0.f, 0.f};
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float x0 = fmaf(sv[2 * i], sl2, -m_use);
        const float x1 = fmaf(sv[2 * i + 1], sl2, -m_use);
        const float p0 = fast_exp2(x0);
        const float p1 = (i & 1) ? exp2_poly(x1) : fast_exp2(x1);
        sum4[(2 * i) & 3] += p0;
        sum4[(2 * i + 1) & 3] += p1;
        pk[i] = pack_bf16(p0, p1);
      }
      const float sum0 = sum4[0] + sum4[2], sum1 = sum4[1] + sum4[3];
      // P buffer j&1 is free once PV(j-2) has completed.
      if (j >= 2 && !__all_sync(0xffffffffu, mbar_wait(&bars[B_PVDONE + (j & 1)],
                                                        ((j - 2) >> 1) & 1))) {
        failed = true;
        continue;
      }
      // O may only be rescaled while no PV is in flight: after PV(j-1).
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&bars[B_PVDONE + ((j - 1) & 1)],
                                               ((j - 1) >> 1) & 1))) {
          failed = true;
          continue;
        }
        tc_fence_after();
#pragma unroll
        for (int cb = 0; cb < 4; ++cb) {
          uint32_t orow[16];
          tmem_ld16(t_o + cb * 16, orow);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
          tmem_st16(t_o + cb * 16, orow);
        }
      }
      tc_fence_after();
      const uint32_t t_p = t_p0 + (uint32_t)(j & 1) * 64u;
      tmem_st16(t_p, pk);
      tmem_st16(t_p + 16, pk + 16);
      tmem_wait_st();
      l_run = l_run * alpha + (sum0 + sum1);
      m_run = m_use;
      tc_fence_before();
      mbar_arrive(&bars[B_PREADY + (j & 1)]);
    }
    // epilogue: combine the two halves' row sums, then each half stores its
    // 64 output columns
    bool stop = failed || *abort_flag != 0;
    if (!stop)
      stop = !mbar_wait(&bars[B_PVDONE + ((nkv - 1) & 1)], ((nkv - 1) >> 1) & 1);
    stop = __any_sync(0xffffffffu, stop);
    if (!stop) red[(4 + wg) * 128 + row_in_tile] = l_run;
    if (!named_bar_any(1, 256, stop)) {
      tc_fence_after();
      const float l_tot = l_run + red[(4 + (wg ^ 1)) * 128 + row_in_tile];
      const int row = q_tile * kRows + row_in_tile;
      const float inv_l = 1.f / l_tot;
      uint32_t orow[64];
      tmem_ld32(t_o + 0, orow);
      tmem_ld32(t_o + 32, orow + 32);
      tmem_wait_ld();
      if (row < p.S) {
        __nv_bfloat16* dst = p.o + (int64_t)b * p.os_b + (int64_t)row * p.os_s +
                             (int64_t)h * p.os_h + wg * 64;
        uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 v;
          v.x = pack_bf16(__uint_as_float(orow[c * 8 + 0]) * inv_l,
                          __uint_as_float(orow[c * 8 + 1]) * inv_l);
          v.y = pack_bf16(__uint_as_float(orow[c * 8 + 2]) * inv_l,
                          __uint_as_float(orow[c * 8 + 3]) * inv_l);
          v.z = pack_bf16(__uint_as_float(orow[c * 8 + 4]) * inv_l,
                          __uint_as_float(orow[c * 8 + 5]) * inv_l);
          v.w = pack_bf16(__uint_as_float(orow[c * 8 + 6]) * inv_l,
                          __uint_as_float(orow[c * 8 + 7]) * inv_l);
          d4[c] = v;
        }
        if (wg == 0)
          p.lse[((int64_t)b * p.H + h) * p.S + row] =
              (m_run + __log2f(l_tot)) * 0.69314718055994531f;
      }
    } else {
      *abort_flag = 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace fwd

int launch_attn_fwd_bf16(const AttnShape& sh, int kv_len, const fa_tensor_t* q,
                         const fa_tensor_t* k, const fa_tensor_t* v,
                         const fa_tensor_t* o, float* lse, float scale,
                         cudaStream_t stream) {
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_bshd(&tq, q, sh.B, sh.S, sh.H, sh.D, 128);
  if (rc) return rc;
  rc = make_tmap_bshd(&tk, k, sh.B, kv_len, sh.H, sh.D, 128);
  if (rc) return rc;
  rc = make_tmap_bshd(&tv, v, sh.B, kv_len, sh.H, sh.D, 128);
  if (rc) return rc;
  fwd::Params p;
  p.S = sh.S;
  p.H = sh.H;
  p.kv_len = kv_len;
  p.nkv = (kv_len + fwd::kKeys - 1) / fwd::kKeys;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.o = reinterpret_cast<__nv_bfloat16*>(o->data);
  p.os_b = o->stride_b;
  p.os_s = o->stride_s;
  p.os_h = o->stride_h;
  p.lse = lse;
  rc = ensure_smem_attr((const void*)fwd::attn_fwd_kernel, fwd::kSmemBytes,
                        kKernelFwdBf16);
  if (rc) return rc;
  dim3 grid((sh.S + fwd::kRows - 1) / fwd::kRows, sh.H, sh.B);
  fwd::attn_fwd_kernel<<<grid, fwd::kThreads, fwd::kSmemBytes, stream>>>(
      tq, tk, tv, p);
  return launch_status();
}

}  // namespace fa
