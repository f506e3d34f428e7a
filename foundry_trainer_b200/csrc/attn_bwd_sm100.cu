// attn_bwd_sm100.cu — bf16 joint-attention backward for sm_100a.
//
// Gradient of O = softmax(Q K^T * scale) V, the hand-written backward of the
// reference op (crates/foundry-spike/src/lib.rs:216-263):
//   P   = exp(S*scale - LSE)              (recomputed from the saved LSE)
//   dV  = P^T dO                          (lib.rs:244)
//   dP  = dO V^T                          (lib.rs:243)
//   dS  = P * (dP - Delta),  Delta = rowsum(dO * O)   (= rowsum(dP*P), lib.rs:246-250)
//   dQ  = scale * dS K,  dK = scale * dS^T Q          (lib.rs:252-257)
// The reference forms dS in fp32 and runs dQ/dK as fp32 GEMMs; here dS is
// rounded to bf16 for the tensor core with fp32 accumulation.
//
// One CTA owns one 128-key K/V tile of one (b, h) and walks all 128-row Q
// tiles (K/V stationary), starting at Q tile `kv_tile` and wrapping, so the
// CTAs of one head add into different dQ rows at any moment instead of all
// contending for the same L2 lines. 14 warps:
//   warp 8        TMA producer: K, V once; Q_i, dO_i, LSE_i, Delta_i per step
//   warp 9        tcgen05 MMA issuer (the whole warp runs the loop, one
//                 elected lane issues), TMEM owner
//   warps 0-3     softmax backward for queries 0-63 of the tile (one key row
//                 per thread); dV epilogue
//   warps 10-13   the same for queries 64-127; dK epilogue
//   warps 4-7     dQ drain: dQ^T from TMEM, staged row-major (query, d) in
//                 the step's own Q_i|dO_i slot (64 KB, free once the dQ^T MMA
//                 has completed), added into dq_acc (B, H, S_pad, D) with TMA
//                 bulk reduce-adds (fp32) — or, in deterministic mode, stored
//                 to this CTA's own partial slot with bulk copies; the slot
//                 goes back to the producer when the bulk ops have read it
// TMEM (512 columns):
//   A [0,128)    S^T_i; after the softmax, per query half h (columns
//                64h..64h+63): P^T (bf16 pairs, 32 columns) then dS^T (32
//                columns) — each half only overwrites columns it has read
//   B [128,256)  dP^T_i, then dQ^T_i = K^T dS^T_i (fp32; lane = head-dim
//                column, column = query)
//   dV [256,384) dK [384,512)   accumulators over all Q tiles
// tcgen05.mma operations issued by one thread execute in issue order, so an
// MMA that overwrites columns an earlier MMA reads needs no wait; TMEM read by
// the softmax or the drain is handed back through barriers. dQ_i is drained
// while S^T_{i+1} runs, and TMEM B is handed
// back (DQFREE) as soon as it has been read into registers. The dS^T tile is
// free for the next step's softmax once the dQ^T MMA has read it (DSFREE).
#include "attn_common.h"
#include "rope.cuh"
#include "sm100_ptx.cuh"

namespace fa {
namespace bwd {

constexpr int kRows = 128;
constexpr int kTileBytes = 32768;
constexpr int kBlkBytes = 16384;
constexpr int kThreads = 448;

constexpr int kOffK = 0;
constexpr int kOffV = kOffK + kTileBytes;
// two stages of [Q_i | dO_i] (64 KB each, contiguous: the dQ_i staging area
// once the step's MMAs are done)
constexpr int kOffStage = kOffV + kTileBytes;
constexpr int kStageBytes = 2 * kTileBytes;
constexpr int kOffDS = kOffStage + 2 * kStageBytes;
constexpr int kOffLse = kOffDS + kTileBytes;    // 2 x 512 B
constexpr int kOffDelta = kOffLse + 1024;       // 2 x 512 B
constexpr int kOffBar = kOffDelta + 1024;
constexpr int kNumBars = 16;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 64;

constexpr int B_KV = 0;
constexpr int B_QFULL = 1;    // + stage
constexpr int B_QEMPTY = 3;   // + stage
constexpr int B_SDP = 5;
constexpr int B_PS = 6;
constexpr int B_DQFULL = 7;
constexpr int B_DQFREE = 8;
constexpr int B_FINAL = 10;
constexpr int B_DSFREE = 11;
constexpr int B_DSREADY = 12;  // dS^T_i copied to shared memory (drain warps)

constexpr uint32_t kColA = 0;
constexpr uint32_t kColB = 128;
constexpr uint32_t kColDV = 256;
constexpr uint32_t kColDK = 384;

struct Params {
  int S, H, kv_len, nq, s_pad;
  float scale, scale_log2;
  const float* lse2_pad;    // (B, H, s_pad): LSE * log2(e), +inf padding
  const float* delta_pad;   // (B, H, s_pad): rowsum(dO*O), 0 padding
  // dK / dV output: bf16 strided tensors (acc 0), fp32 (B, kv_len, H, D)
  // buffers that the result is added to (acc 1) or stored in (acc 2), or
  // fp32 rows stored per key segment (acc 3: row j to seg_dk[j / seg] at
  // local row j % seg, (B, seg, H, D) each; a segment may be a peer GPU's
  // memory, written with plain stores)
  int acc;
  int seg;
  float* seg_dk[FA_PEER_MAX];
  float* seg_dv[FA_PEER_MAX];
  __nv_bfloat16* dk;
  int64_t dks_b, dks_s, dks_h;
  __nv_bfloat16* dv;
  int64_t dvs_b, dvs_s, dvs_h;
  float* dk_acc;            // (B, kv_len, H, D) fp32
  float* dv_acc;
  float* dq_acc;            // (B, H, s_pad, D) fp32, zeroed by the caller
  // Deterministic mode (dq_acc unused): the CTA of K/V tile t stores its
  // contribution to each dQ tile into its own slot t of the fp32
  // (n_kv_tiles, B, H, s_pad, D) array; a later pass sums the slots in index
  // order, so repeated runs give the same bits. nullptr: reduce-adds.
  float* dq_part;
  RopeArgs rope;            // rope.pos == nullptr: no rotation
  // acc 0: 1 = dK / dV leave through TMA tile stores (tm_dk, tm_dv), staged
  // in the K and V tiles' shared memory (free once the last MMA completed);
  // 0 = plain stores from registers (a layout the tensor maps cannot encode)
  int tma_out;
};

// Q tile visited at step i by the CTA of K/V tile `kv_tile`.
__device__ __forceinline__ int q_tile_of(int i, int kv_tile, int nq) {
  const int t = i + kv_tile % nq;
  return t >= nq ? t - nq : t;
}

// dst[0 .. bytes/4) += src[...] (fp32), performed by the TMA unit.
__device__ __forceinline__ void bulk_reduce_add_f32(float* dst, const float* src,
                                                    uint32_t bytes) {
  asm volatile(
      "cp.reduce.async.bulk.global.shared::cta.bulk_group.add.f32 [%0], [%1], %2;" ::"l"(
          dst),
      "r"(smem_u32(src)), "r"(bytes)
      : "memory");
}

// dst[0 .. bytes/4) = src[...], performed by the TMA unit.
__device__ __forceinline__ void bulk_store_f32(float* dst, const float* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src,
                                          uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes "
      "[%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// fp32 output row of key `key` (acc 1-3): the accumulator, or the key's
// segment buffer (acc 3).
__device__ __forceinline__ float* f32_row(const Params& p, bool is_dk, int b, int key, int h) {
  float* base;
  int64_t row;
  if (p.acc == 3) {
    const int o = key / p.seg;
    base = is_dk ? p.seg_dk[o] : p.seg_dv[o];
    row = (int64_t)b * p.seg + (key - o * p.seg);
  } else {
    base = is_dk ? p.dk_acc : p.dv_acc;
    row = (int64_t)b * p.kv_len + key;
  }
  return base + (row * p.H + h) * 128;
}

// Writes columns [col0, col0+32) of the 32 fp32 rows a warp holds (lane =
// row, v = the lane's 32 values) through a 4 KB shared slab: each row goes
// in as 8 float4 (column c at c ^ (row & 7), no bank conflicts), and comes
// out as 4 whole rows of 128 contiguous bytes per store instruction, so a
// segment in another GPU's memory receives full lines over NVLink.
__device__ __forceinline__ void store_rows32_f32(const Params& p, bool is_dk, int b, int key0,
                                                 int h, int col0, const float* v,
                                                 float4* slab, int lane) {
#pragma unroll
  for (int c = 0; c < 8; ++c)
    slab[lane * 8 + (c ^ (lane & 7))] =
        make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
  __syncwarp();
  const int cc = lane & 7;
  // The warp's 32 rows are consecutive rows of one buffer unless a segment
  // boundary falls among them: their addresses then follow from the first
  // row's (the per-row segment division and parameter lookup measured 40% of
  // the epilogue at the sequence-parallel shard shape). Warp-uniform branch.
  const int last = min(key0 + 31, p.kv_len - 1);
  if (key0 < p.kv_len && (p.acc != 3 || key0 / p.seg == last / p.seg)) {
    float* row0 = f32_row(p, is_dk, b, key0, h) + col0;
    const int64_t rstride = (int64_t)p.H * 128;
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int rr = it * 4 + (lane >> 3);
      float4 x = slab[rr * 8 + (cc ^ (rr & 7))];
      if (key0 + rr < p.kv_len) {
        float4* dst = reinterpret_cast<float4*>(row0 + rr * rstride) + cc;
        if (p.acc == 1) {
          const float4 a = *dst;
          x.x += a.x;
          x.y += a.y;
          x.z += a.z;
          x.w += a.w;
        }
        *dst = x;
      }
    }
  } else {
#pragma unroll
    for (int it = 0; it < 8; ++it) {
      const int rr = it * 4 + (lane >> 3);
      float4 x = slab[rr * 8 + (cc ^ (rr & 7))];
      const int key = key0 + rr;
      if (key < p.kv_len) {
        float4* dst = reinterpret_cast<float4*>(f32_row(p, is_dk, b, key, h) + col0) + cc;
        if (p.acc == 1) {
          const float4 a = *dst;
          x.x += a.x;
          x.y += a.y;
          x.z += a.z;
          x.w += a.w;
        }
        *dst = x;
      }
    }
  }
  __syncwarp();
}

// Stages columns [32a, 32a+32) of bf16 row `r` of a (128 x 128) tile in
// shared memory in the SWIZZLE_128B layout of the TMA tile store (two 64-
// column blocks; chunk c of row r at c ^ (r & 7): the 32 rows of a warp
// cover all bank groups).
__device__ __forceinline__ void stage_chunk32(uint8_t* tile, int r, int a, const float* v) {
  uint8_t* blk = tile + (a >> 1) * kBlkBytes;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 o;
    o.x = pack_bf16(v[8 * c + 0], v[8 * c + 1]);
    o.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
    o.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
    o.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(blk + sw128_offset(r, (a & 1) * 4 + c)) = o;
  }
}

// Writes columns [col0, col0+32) of one bf16 dK/dV row held in registers.
__device__ __forceinline__ void store_chunk32(const Params& p, bool is_dk, int b,
                                              int key, int h, int col0,
                                              const float* v) {
  __nv_bfloat16* dst =
      (is_dk ? p.dk + (int64_t)b * p.dks_b + (int64_t)key * p.dks_s +
                   (int64_t)h * p.dks_h
             : p.dv + (int64_t)b * p.dvs_b + (int64_t)key * p.dvs_s +
                   (int64_t)h * p.dvs_h) +
      col0;
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 o;
    o.x = pack_bf16(v[8 * c + 0], v[8 * c + 1]);
    o.y = pack_bf16(v[8 * c + 2], v[8 * c + 3]);
    o.z = pack_bf16(v[8 * c + 4], v[8 * c + 5]);
    o.w = pack_bf16(v[8 * c + 6], v[8 * c + 7]);
    d4[c] = o;
  }
}

// (cos, sin) of the 16 frequencies of 32-wide axis `a` for `token`, from the
// table: 128 contiguous bytes, 8 independent 16-byte loads.
__device__ __forceinline__ void load_axis_cs(const RopeArgs& r, int token, int a,
                                             float4* cs) {
  const float4* t4 = reinterpret_cast<const float4*>(
      r.table + (int64_t)(token + r.pos_offset) * (r.n_axes * (r.axis_dim >> 1)) + a * 16);
#pragma unroll
  for (int u = 0; u < 8; ++u) cs[u] = t4[u];
}

// Inverse rotation of one 32-wide axis segment held in v[0..32).
__device__ __forceinline__ void unrotate_axis(const float4* cs, float* v) {
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float4 q = cs[j >> 1];
    const float c = (j & 1) ? q.z : q.x;
    const float sn = (j & 1) ? q.w : q.y;
    const float x1 = v[j];
    const float x2 = v[j + 16];
    v[j] = __fadd_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    v[j + 16] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(-x1, sn));
  }
}

__global__ void __launch_bounds__(kThreads, 1)
attn_bwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v,
                const __grid_constant__ CUtensorMap tm_do,
                const __grid_constant__ CUtensorMap tm_dk,
                const __grid_constant__ CUtensorMap tm_dv, const __grid_constant__ Params p) {
  extern __shared__ __align__(1024) uint8_t smem[];
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  // The layout needs a 1024-byte aligned window (SWIZZLE_128B atoms).
  if ((smem_u32(smem) & 1023u) != 0) {
    if (threadIdx.x == 0) report_status(2 /* FA_ERR_UNSUPPORTED */);
    return;
  }

  const int warp = warp_id();
  const int lane = lane_id();
  const int kv_tile = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int nq = p.nq;

  if (threadIdx.x == 0) {
    mbar_init(&bars[B_KV], 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars[B_QFULL + s], 1);
      mbar_init(&bars[B_QEMPTY + s], 1);
    }
    mbar_init(&bars[B_SDP], 1);
    mbar_init(&bars[B_PS], 256);
    mbar_init(&bars[B_DQFULL], 1);
    mbar_init(&bars[B_DQFREE], 128);
    mbar_init(&bars[B_FINAL], 1);
    mbar_init(&bars[B_DSFREE], 1);
    mbar_init(&bars[B_DSREADY], 128);
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
  const int64_t lse_row0 = ((int64_t)b * p.H + h) * p.s_pad;

  if (warp == 8) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      tma_prefetch_desc(&tm_do);
      const int krow = kv_tile * kRows;
      mbar_arrive_expect_tx(&bars[B_KV], 2 * kTileBytes);
      tma_load_4d(smem + kOffK, &tm_k, &bars[B_KV], 0, krow, h, b);
      tma_load_4d(smem + kOffK + kBlkBytes, &tm_k, &bars[B_KV], 64, krow, h, b);
      tma_load_4d(smem + kOffV, &tm_v, &bars[B_KV], 0, krow, h, b);
      tma_load_4d(smem + kOffV + kBlkBytes, &tm_v, &bars[B_KV], 64, krow, h, b);
      bool ok = true;
      for (int i = 0; i < nq; ++i) {
        const int st = i & 1, n = i >> 1;
        if (*abort_flag) break;
        if (i >= 2 && !(ok = mbar_wait(&bars[B_QEMPTY + st], (n - 1) & 1)))
          break;
        const int qrow = q_tile_of(i, kv_tile, nq) * kRows;
        uint64_t* bar = &bars[B_QFULL + st];
        mbar_arrive_expect_tx(bar, 2 * kTileBytes + 1024);
        uint8_t* qd = smem + kOffStage + st * kStageBytes;
        uint8_t* dd = qd + kTileBytes;
        tma_load_4d(qd, &tm_q, bar, 0, qrow, h, b);
        tma_load_4d(qd + kBlkBytes, &tm_q, bar, 64, qrow, h, b);
        tma_load_4d(dd, &tm_do, bar, 0, qrow, h, b);
        tma_load_4d(dd + kBlkBytes, &tm_do, bar, 64, qrow, h, b);
        bulk_load(smem + kOffLse + st * 512, p.lse2_pad + lse_row0 + qrow, 512,
                  bar);
        bulk_load(smem + kOffDelta + st * 512, p.delta_pad + lse_row0 + qrow,
                  512, bar);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 9) {
    // ---------------------------------------- MMA issuer (whole warp, one lane issues)
    {
      constexpr uint32_t kIdKK = idesc_bf16(128, 128, false, false);
      constexpr uint32_t kIdKM = idesc_bf16(128, 128, false, true);
      constexpr uint32_t kIdMM = idesc_bf16(128, 128, true, true);
      const uint32_t k_base = smem_u32(smem + kOffK);
      const uint32_t v_base = smem_u32(smem + kOffV);
      const uint32_t ds_base = smem_u32(smem + kOffDS);
      bool ok = mbar_wait_w(&bars[B_KV], 0);
      tc_fence_after();
      for (int i = 0; ok && i < nq; ++i) {
        const int st = i & 1, n = i >> 1;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
        if (!(ok = mbar_wait_w(&bars[B_QFULL + st], n & 1))) break;
        const uint32_t q_base = smem_u32(smem + kOffStage + st * kStageBytes);
        const uint32_t do_base = q_base + kTileBytes;
        // S^T_i = K Q_i^T -> A. A was read by dV/dK of step i-1: tcgen05.mma
        // operations issued by one thread execute in issue order, so no wait.
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss_w(tmem + kColA, kmajor_desc(k_base, kk, kBlkBytes),
                    kmajor_desc(q_base, kk, kBlkBytes), kIdKK, kk > 0);
        // dP^T_i = V dO_i^T -> B   (B held dQ_{i-1} until the drain read it)
        if (i > 0 && !(ok = mbar_wait_w(&bars[B_DQFREE], (i - 1) & 1))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss_w(tmem + kColB, kmajor_desc(v_base, kk, kBlkBytes),
                    kmajor_desc(do_base, kk, kBlkBytes), kIdKK, kk > 0);
        umma_commit_w(&bars[B_SDP]);
        if (!(ok = mbar_wait_w(&bars[B_PS], i & 1))) break;
        tc_fence_after();
        // dV += P^T dO_i ; dK += dS^T Q_i   (A operands from TMEM; K slice kk
        // is queries 16kk..16kk+15: half kk>>2, eight packed columns each)
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts_w(tmem + kColDV, tmem + kColA + (kk >> 2) * 64 + (kk & 3) * 8,
                    mnmajor_desc(do_base, kk, kBlkBytes), kIdKM,
                    (i > 0 || kk > 0) ? 1u : 0u);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts_w(tmem + kColDK,
                    tmem + kColA + (kk >> 2) * 64 + 32 + (kk & 3) * 8,
                    mnmajor_desc(q_base, kk, kBlkBytes), kIdKM,
                    (i > 0 || kk > 0) ? 1u : 0u);
        // dQ^T_i = K^T dS^T_i -> B   (both operands MN-major in shared memory;
        // dS^T_i reaches shared memory while dV/dK run)
        if (!(ok = mbar_wait_w(&bars[B_DSREADY], i & 1))) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss_w(tmem + kColB, mnmajor_desc(k_base, kk, kBlkBytes),
                    mnmajor_desc(ds_base, kk, kBlkBytes), kIdMM, kk > 0);
        umma_commit_w(&bars[B_DQFULL]);
        umma_commit_w(&bars[B_DSFREE]);
      }
      if (!ok && lane == 0) *abort_flag = 1;
      umma_commit_w(&bars[B_FINAL]);
      mbar_wait(&bars[B_FINAL], 0);
    }
  } else if (warp < 4 || warp >= 10) {
    // ------------------------------- softmax backward (key rows, query half)
    const int half = warp >= 10 ? 1 : 0;
    const int sub = warp & 3;
    const int key_in_tile = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t t_a = tmem + lane_off + kColA + (uint32_t)half * 64u;
    const uint32_t t_b = tmem + lane_off + kColB + (uint32_t)half * 64u;
    const float sl2 = p.scale_log2;
    const uint64_t sl2_2 = f2_pack(sl2, sl2);
    bool ok = true;
    for (int i = 0; i < nq; ++i) {
      const int st = i & 1, n = i >> 1;
      if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_SDP], i & 1));
      if (!ok) break;
      // the LSE / Delta slices arrived with Q_i (already complete here)
      ok = __all_sync(0xffffffffu, mbar_wait(&bars[B_QFULL + st], n & 1));
      if (!ok) break;
      tc_fence_after();
      const float4* lse4 =
          reinterpret_cast<const float4*>(smem + kOffLse + st * 512) + half * 16;
      const float4* dlt4 =
          reinterpret_cast<const float4*>(smem + kOffDelta + st * 512) + half * 16;
      // This half's S^T columns 32-63 are read first: dS^T (columns 32-63)
      // is written over them; P^T of chunk c goes over columns 8c..8c+7,
      // which chunk c or an earlier chunk has already read.
      uint32_t s_hi[32];
      tmem_ld32(t_a + 32, s_hi);
#pragma unroll
      for (int cb = 0; cb < 4; ++cb) {
        uint32_t dr[16], s_lo[16];
        if (cb < 2) tmem_ld16(t_a + cb * 16, s_lo);
        tmem_ld16(t_b + cb * 16, dr);
        tmem_wait_ld();
        const uint32_t* sr = cb < 2 ? s_lo : s_hi + (cb - 2) * 16;
        uint32_t pk[8], dk[8];
        // pairs of columns through the packed fp32x2 pipe (each lane rounds
        // as the scalar instruction would): x = S*scale*log2e - LSE2,
        // P = 2^x, dS = P * (dP - Delta)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 l = lse4[cb * 4 + u];
          const float4 dl = dlt4[cb * 4 + u];
          const int c = 4 * u;
          float x0, x1, x2, x3;
          f2_unpack(ffma2(f2_pack(__uint_as_float(sr[c + 0]), __uint_as_float(sr[c + 1])),
                          sl2_2, f2_pack(-l.x, -l.y)), x0, x1);
          f2_unpack(ffma2(f2_pack(__uint_as_float(sr[c + 2]), __uint_as_float(sr[c + 3])),
                          sl2_2, f2_pack(-l.z, -l.w)), x2, x3);
          const float p0 = fast_exp2(x0), p1 = fast_exp2(x1);
          const float p2 = fast_exp2(x2), p3 = fast_exp2(x3);
          pk[2 * u] = pack_bf16(p0, p1);
          pk[2 * u + 1] = pack_bf16(p2, p3);
          float d0, d1, d2, d3;
          f2_unpack(fmul2(f2_pack(p0, p1),
                          fsub2(f2_pack(__uint_as_float(dr[c + 0]), __uint_as_float(dr[c + 1])),
                                f2_pack(dl.x, dl.y))), d0, d1);
          f2_unpack(fmul2(f2_pack(p2, p3),
                          fsub2(f2_pack(__uint_as_float(dr[c + 2]), __uint_as_float(dr[c + 3])),
                                f2_pack(dl.z, dl.w))), d2, d3);
          dk[2 * u] = pack_bf16(d0, d1);
          dk[2 * u + 1] = pack_bf16(d2, d3);
        }
        tmem_st8(t_a + cb * 8, pk);       // P^T: columns 64h + [0, 32)
        tmem_st8(t_a + 32 + cb * 8, dk);  // dS^T: columns 64h + [32, 64)
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars[B_PS]);
    }
    // epilogue: warps 0-3 store dV, warps 10-13 store dK (scaled, and
    // un-rotated when the op owns the RoPE), one 32-column axis at a time
    // (fp32 outputs through per-warp 4 KB slabs of the dS^T tile, free once
    // the last MMA has completed);
    // the (cos, sin) of the next axis are loaded while this one is stored,
    // the first before the wait for the last MMA
    const bool is_dk = half == 1;
    const int key = kv_tile * kRows + key_in_tile;
    const bool unrot = is_dk && p.rope.pos != nullptr && p.rope.table != nullptr &&
                       key < p.kv_len;
    float4 cs[8], cs_next[8];
    if (unrot) load_axis_cs(p.rope, key, 0, cs);
    const bool tma_out = p.acc == 0 && p.tma_out;
    uint8_t* out_tile = smem + (is_dk ? kOffK : kOffV);
    const bool good = ok && __all_sync(0xffffffffu, mbar_wait(&bars[B_FINAL], 0)) &&
                      !__any_sync(0xffffffffu, *abort_flag != 0);
    if (good) {
      tc_fence_after();
      const uint32_t t_acc = tmem + lane_off + (is_dk ? kColDK : kColDV);
#pragma unroll
      for (int a = 0; a < 4; ++a) {
        uint32_t r[32];
        tmem_ld32(t_acc + a * 32, r);
        if (unrot && a < 3) load_axis_cs(p.rope, key, a + 1, cs_next);
        tmem_wait_ld();
        float* v = reinterpret_cast<float*>(r);
        if (is_dk) {
#pragma unroll
          for (int c = 0; c < 32; ++c) v[c] *= p.scale;
          if (unrot) unrotate_axis(cs, v);
        }
        if (p.acc)
          store_rows32_f32(p, is_dk, b, kv_tile * kRows + sub * 32, h, a * 32, v,
                           reinterpret_cast<float4*>(smem + kOffDS + (half * 4 + sub) * 4096),
                           lane);
        else if (tma_out)
          stage_chunk32(out_tile, key_in_tile, a, v);
        else if (key < p.kv_len)
          store_chunk32(p, is_dk, b, key, h, a * 32, v);
        if (unrot && a < 3) {
#pragma unroll
          for (int u = 0; u < 8; ++u) cs[u] = cs_next[u];
        }
      }
    } else {
      *abort_flag = 1;
    }
    if (tma_out) {
      // the warpgroup's tile (rows past kv_len are clipped by the tensor map)
      fence_proxy_async_smem();
      const bool stop = half ? named_bar_any(4, 128, !good) : named_bar_any(3, 128, !good);
      if (!stop && sub == 0 && lane == 0) {
        const CUtensorMap* map = is_dk ? &tm_dk : &tm_dv;
        tma_store_4d(map, out_tile, 0, kv_tile * kRows, h, b);
        tma_store_4d(map, out_tile + kBlkBytes, 64, kv_tile * kRows, h, b);
        bulk_commit_group();
        bulk_wait_group_read0();  // shared memory read before the CTA exits
      }
    }
  } else {
    // ------------------------------ dQ drain (head-dim column per thread)
    const int sub = warp & 3;
    const int d = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t t_b = tmem + lane_off + kColB;
    const bool leader = (warp == 4 && lane == 0);
    const int64_t bh_rows = ((int64_t)b * p.H + h) * p.s_pad;
    float* dq_bh = p.dq_part != nullptr
                       ? p.dq_part + ((int64_t)kv_tile * gridDim.z * p.H * p.s_pad + bh_rows) * 128
                       : p.dq_acc + bh_rows * 128;
    // a thread writes column d of 64 query rows; a warp 128 contiguous bytes
    auto stage = [&](float* buf, const uint32_t* v) {
#pragma unroll
      for (int j = 0; j < 64; ++j) buf[j * 128 + d] = __uint_as_float(v[j]);
    };
    // dS^T copy: this thread's key row (lane quarter of the warp), both query
    // halves: 32 packed columns each, stored as 16-byte chunks 0-7 of swizzle
    // block h (the MN-major B operand of the dQ^T MMA)
    const uint32_t t_ds = tmem + lane_off + kColA + 32;
    const int key_row = sub * 32 + lane;
    int reduce_pending = -1;  // slot whose bulk reduces the leader has not yet seen read
    for (int i = 0; i < nq; ++i) {
      // dS^T_i: the softmax wrote it to TMEM (PS); the dQ^T MMA of step i-1
      // has finished reading the shared tile (DSFREE)
      {
        bool stop = *abort_flag != 0;
        if (!stop) stop = !mbar_wait(&bars[B_PS], i & 1);
        if (!stop && i > 0) stop = !mbar_wait(&bars[B_DSFREE], (i - 1) & 1);
        if (named_bar_any(2, 128, stop)) break;
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          uint32_t dsr[32];
          tmem_ld32(t_ds + hh * 64, dsr);
          tmem_wait_ld();
          uint8_t* blk = smem + kOffDS + hh * kBlkBytes;
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(blk + sw128_offset(key_row, u)) =
                make_uint4(dsr[4 * u], dsr[4 * u + 1], dsr[4 * u + 2], dsr[4 * u + 3]);
        }
        fence_proxy_async_smem();
        tc_fence_before();
        mbar_arrive(&bars[B_DSREADY]);
      }
      // the previous step's reduces have had a whole dS copy to read their slot
      if (leader && reduce_pending >= 0) {
        bulk_wait_group_read0();
        mbar_arrive(&bars[B_QEMPTY + reduce_pending]);
        reduce_pending = -1;
      }
      // leave together: the staging uses a named barrier over warps 4-7
      bool stop = *abort_flag != 0;
      if (!stop) stop = !mbar_wait(&bars[B_DQFULL], i & 1);
      if (named_bar_any(2, 128, stop)) break;
      tc_fence_after();
      const int st = i & 1;
      // the step's Q_i | dO_i slot: every MMA reading it completed before DQFULL
      float* buf = reinterpret_cast<float*>(smem + kOffStage + st * kStageBytes);
      float* dst = dq_bh + (int64_t)q_tile_of(i, kv_tile, nq) * kRows * 128;
      uint32_t r[64];
      tmem_ld32(t_b + 0, r);
      tmem_ld32(t_b + 32, r + 32);
      tmem_wait_ld();
      stage(buf, r);
      tmem_ld32(t_b + 64, r);
      tmem_ld32(t_b + 96, r + 32);
      tmem_wait_ld();
      // TMEM B can take dP^T_{i+1}
      tc_fence_before();
      mbar_arrive(&bars[B_DQFREE]);
      stage(buf + 64 * 128, r);
      fence_proxy_async_smem();
      named_bar_sync(2, 128);
      if (leader) {
        if (p.dq_part != nullptr) {
          bulk_store_f32(dst, buf, 32768);
          bulk_store_f32(dst + 64 * 128, buf + 64 * 128, 32768);
        } else {
          bulk_reduce_add_f32(dst, buf, 32768);
          bulk_reduce_add_f32(dst + 64 * 128, buf + 64 * 128, 32768);
        }
        bulk_commit_group();
        reduce_pending = st;  // slot handed back once the reduces have read it
      }
    }
    if (leader && reduce_pending >= 0) {
      bulk_wait_group_read0();
      mbar_arrive(&bars[B_QEMPTY + reduce_pending]);
    }
    if (leader) bulk_wait_group0();  // reductions complete before exit
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace bwd

int launch_attn_bwd_bf16(const AttnShape& sh, int kv_len, const fa_tensor_t* q,
                         const fa_tensor_t* k, const fa_tensor_t* v,
                         const fa_tensor_t* d_o, const float* lse2_pad,
                         const float* delta_pad, float* dq_acc,
                         const fa_tensor_t* dk, const fa_tensor_t* dv,
                         float* dk_acc, float* dv_acc, int accumulate, float scale,
                         const fa_rope_t* rope, const float2* rope_table,
                         cudaStream_t stream, const BwdScatter* scatter, float* dq_part) {
  if (rope != nullptr && (rope->axis_dim != 32 || rope->n_axes != 4))
    return FA_ERR_UNSUPPORTED;  // the dK epilogue un-rotates 32-wide axes
  if (rope != nullptr && rope_table == nullptr)
    return FA_ERR_INVALID_ARG;  // ... with the (cos, sin) table
  CUtensorMap tq, tk, tv, tdo, tdk, tdv;
  int rc = make_tmap_bshd(&tq, q, sh.B, sh.S, sh.H, sh.D, 128);
  if (!rc) rc = make_tmap_bshd(&tk, k, sh.B, kv_len, sh.H, sh.D, 128);
  if (!rc) rc = make_tmap_bshd(&tv, v, sh.B, kv_len, sh.H, sh.D, 128);
  if (!rc) rc = make_tmap_bshd(&tdo, d_o, sh.B, sh.S, sh.H, sh.D, 128);
  if (rc) return rc;
  bwd::Params p;
  p.S = sh.S;
  p.H = sh.H;
  p.kv_len = kv_len;
  p.nq = (sh.S + 127) / 128;
  p.s_pad = p.nq * 128;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse2_pad = lse2_pad;
  p.delta_pad = delta_pad;
  p.acc = (dk_acc != nullptr) ? (accumulate ? 1 : 2) : 0;
  p.seg = 1;
  for (int i = 0; i < FA_PEER_MAX; ++i) p.seg_dk[i] = p.seg_dv[i] = nullptr;
  if (scatter != nullptr) {
    p.acc = 3;
    p.seg = scatter->seg;
    for (int i = 0; i < scatter->n; ++i) {
      p.seg_dk[i] = scatter->dk[i];
      p.seg_dv[i] = scatter->dv[i];
    }
  }
  p.dk = dk ? reinterpret_cast<__nv_bfloat16*>(dk->data) : nullptr;
  p.dks_b = dk ? dk->stride_b : 0;
  p.dks_s = dk ? dk->stride_s : 0;
  p.dks_h = dk ? dk->stride_h : 0;
  p.dv = dv ? reinterpret_cast<__nv_bfloat16*>(dv->data) : nullptr;
  p.dvs_b = dv ? dv->stride_b : 0;
  p.dvs_s = dv ? dv->stride_s : 0;
  p.dvs_h = dv ? dv->stride_h : 0;
  p.dk_acc = dk_acc;
  p.dv_acc = dv_acc;
  p.dq_acc = dq_acc;
  p.dq_part = dq_part;
  p.rope = make_rope_args(rope);
  p.rope.table = rope_table;
  // bf16 dK / dV through TMA tile stores when both layouts encode (else the
  // maps are copies of tk / tv and are never used)
  p.tma_out = p.acc == 0 && dk != nullptr && dv != nullptr &&
              make_tmap_bshd(&tdk, dk, sh.B, kv_len, sh.H, sh.D, 128) == FA_OK &&
              make_tmap_bshd(&tdv, dv, sh.B, kv_len, sh.H, sh.D, 128) == FA_OK;
  if (!p.tma_out) {
    tdk = tk;
    tdv = tv;
  }
  rc = ensure_smem_attr((const void*)bwd::attn_bwd_kernel, bwd::kSmemBytes,
                        kKernelBwdBf16);
  if (rc) return rc;
  dim3 grid((kv_len + 127) / 128, sh.H, sh.B);
  bwd::attn_bwd_kernel<<<grid, bwd::kThreads, bwd::kSmemBytes, stream>>>(
      tq, tk, tv, tdo, tdk, tdv, p);
  return launch_status();
}

int bwd_device_status() { return tu_device_status(); }

}  // namespace fa
