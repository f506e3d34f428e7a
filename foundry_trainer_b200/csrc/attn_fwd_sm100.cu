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
// One CTA owns two 128-row Q tiles (256 query rows) of one (b, h) and streams
// 128-key K and V tiles through one TMA ring of five slots, in the order they
// are consumed (K_j, V_j, K_{j+1}, ...), so every K/V tile brought into shared
// memory feeds two tiles of tensor-core work and a V tile is requested about
// two steps before its first use (the loads share shared-memory bandwidth
// with the tensor core and take several microseconds to land). The CTAs of a head start at
// different K/V tiles and wrap (the online softmax is order-independent), so
// they do not all request the same tile from L2 at once.
//   warps 0-3   softmax of Q tile 0: one thread per row, the whole 128-key
//               row of S in registers; O rescale (rare) and the epilogue
//   warps 4-7   the same for Q tile 1
//   warp 8      TMA producer of Q0, Q1, K and V (one lane)
//   warp 9      tcgen05 MMA issuer (the whole warp runs the loop, one
//               elected lane issues), TMEM owner
//   warps 10-11 RoPE inside the op: rotate a K tile that arrived unrotated
//               (idle otherwise)
// With RoPE inside the op (the reference's apply_rope on q and k,
// crates/foundry-spike/src/lib.rs:122-129, fused into the tile loads), every
// Q and K tile is rotated once, in shared memory, by the CTA that loads it
// first: at CTA start softmax warpgroup t rotates Q tile t and this CTA's
// own K tile t (the first two K tiles it visits; over all CTAs of a head,
// every K tile), stores them to q_rot / k_rot with TMA (the backward reads
// them) and publishes the K tiles with a state per (b, h, K tile): 0 the
// owning CTA has not started, 1 it is running, 2 the rotated tile is in
// k_rot. The producer loads every other K tile from k_rot when its state is
// 2, waits for a running owner to publish (bounded, ~20 us) when it is 1,
// and otherwise loads it unrotated for warps 10-11 to rotate in its slot;
// no CTA waits on a CTA that has not started, nor unboundedly on any.
// The (cos, sin) pairs come from a packed bf16 table (one 32-bit word per
// token and frequency); a Q tile and the K tile of the same tokens are
// rotated in one pass over the table.
// TMEM (512 columns): S0 [0,128) S1 [128,256) O0 [256,384) O1 [384,512).
// P_t (bf16, two per column) is written over the first 64 columns of S_t
// once the row of S_t is in registers; it is the TMEM A operand of
// O_t += P_t V. The tensor core alternates between the two tiles:
//   S0(j) S1(j) | PV0(j) S0(j+1) | PV1(j) S1(j+1) | PV0(j+1) S0(j+2) ...
// so the softmax of one tile runs while the tensor core works on the other.
#include "attn_common.h"
#include "sm100_ptx.cuh"

namespace fa {
namespace fwd {

constexpr int kRows = 128;          // rows per Q tile
constexpr int kTiles = 2;           // Q tiles per CTA
constexpr int kKeys = 128;          // keys per K/V tile
constexpr int kTileBytes = 32768;   // 128 x 128 bf16
constexpr int kBlkBytes = 16384;    // one 64-column swizzle block
constexpr int kSlots = 5;           // K/V ring: load n (K_j: n = 2j, V_j: 2j+1) in slot n % 5
constexpr int kThreads = 384;

// shared memory map (offsets from a 1024-byte aligned base)
constexpr int kOffQ = 0;  // Q0, Q1; each becomes its tile's O staging at the end
constexpr int kOffKV = kOffQ + kTiles * kTileBytes;
constexpr int kOffBar = kOffKV + kSlots * kTileBytes;
constexpr int kNumBars = 32;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 64 + 1024;  // + alignment slack

// barrier indices
// A ring slot alternates K and V loads (load n goes to slot n % 5), so the
// arrivals of K tiles and of V tiles are signalled on separate barriers: a
// waiter then sees every phase of a barrier it waits on, in order (a parity
// wait that skipped phases could return for the wrong one), and the phase
// of load n is n / 10 for both kinds.
constexpr int B_Q = 0;
constexpr int B_FULL = 1;     // + slot (5): a V tile landed in the slot
constexpr int B_EMPTY = 6;    // + slot (5)
constexpr int B_SFULL = 11;   // + tile: S_t(j) complete
constexpr int B_PREADY = 13;  // + tile: softmax wrote P_t(j) (and rescaled O_t)
constexpr int B_PVDONE = 15;  // + tile: O_t += P_t(j) V_j completed
constexpr int B_FINAL = 17;
constexpr int B_KREADY = 18;  // + slot: the K tile (step >= 2) in the slot is rotated
constexpr int B_QREADY = 23;  // Q tiles and this CTA's own two K tiles rotated (256 arrivals)
constexpr int B_STORED = 24;  // the stores of this CTA's own K tiles have read their slots (2)
constexpr int B_KFULL = 25;   // + slot (5): a K tile landed in the slot
// polling budget for another CTA's published K tile before rotating it here
constexpr long long kPubWaitCycles = 40000;

constexpr uint32_t kColS = 0;    // + 128 t
constexpr uint32_t kColO = 256;  // + 128 t

// Fraction of the exponentials evaluated on the FMA pipe (polynomial)
// instead of MUFU: columns c with (c % kPolyEvery) == kPolyEvery - 1; 0 = none.
// Measured at C2: none 224.7 us, one in eight 235.6 us, one in four 240 us —
// the softmax is bound by instruction issue and latency, not by MUFU.
constexpr int kPolyEvery = 0;
__device__ __forceinline__ constexpr bool poly_column(int c) {
  return kPolyEvery > 0 && c % (kPolyEvery > 0 ? kPolyEvery : 1) == kPolyEvery - 1;
}

// Rotates, in place, the rows of one or two (128 rows x 128 head dims) bf16
// tiles in shared memory laid out as the TMA writes them (two 16 KB
// SWIZZLE_128B blocks of 64 dims each); row r of both tiles is token
// token0 + r (`tb`, when given, is the K tile of the same tokens as the Q
// tile `ta`: the (cos, sin) pairs are read once for both). Rows at or past
// `limit` are the tiles' zero fill and are left alone. Work item (row r,
// axis a, chunk pair u) rotates dims 32a+8u..+7 against 32a+16+8u..+7 with
// frequencies 16a+8u..+7: y1 = x1 c - x2 s, y2 = x2 c + x1 s, each product
// and the sum rounded in fp32 (the reference's separate broadcast_mul and
// add), then rounded to bf16.
// The eight items of a row are eight consecutive lanes (one quarter-warp):
// their 32 (cos, sin) words are the token's 256-byte table row, read as two
// 128-byte runs (`cs` is the packed table, in the order rope_table2_kernel
// writes it: per token, words 4i..4i+3 = frequencies 8i..8i+3 and words
// 32+4i.. = 8i+4..8i+7), and their 16-byte chunk accesses cover the eight
// bank groups of a row — the items of the second 64-dim block take their two
// chunks in the opposite order (x2 first), which the sign of s absorbs:
// out_A = x_A c + x_B s', out_B = x_B c - x_A s' with s' = -s when x_A = x1
// and s' = s when x_A = x2 (the same roundings as y1, y2: a - b = a + (-b)
// and x (-s) = -(x s) exactly). A thread issues the loads of NB items
// before computing them, so one memory latency is exposed per batch.
template <int NB>
__device__ __forceinline__ void rope_rotate_rows(uint8_t* ta, uint8_t* tb, const uint32_t* cs,
                                                 int token0, int limit, int tid, int nthreads) {
  for (int base = tid; base < 1024; base += NB * nthreads) {
    uint4 w[NB][2], xa[NB][2], xb[NB][2];
    bool live[NB];
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      const int task = base + k * nthreads;
      const int r = task >> 3, au = task & 7, a = au >> 1, u = au & 1, hi = a >> 1;
      live[k] = task < 1024 && token0 + r < limit;
      if (live[k]) {
        const uint32_t* row = cs + (int64_t)(token0 + r) * 64;
        w[k][0] = __ldg(reinterpret_cast<const uint4*>(row + 4 * au));
        w[k][1] = __ldg(reinterpret_cast<const uint4*>(row + 32 + 4 * au));
        const int c1 = 4 * (a & 1) + u;
        const uint32_t oA = hi * kBlkBytes + sw128_offset(r, hi ? c1 + 2 : c1);
        const uint32_t oB = hi * kBlkBytes + sw128_offset(r, hi ? c1 : c1 + 2);
        xa[k][0] = *reinterpret_cast<const uint4*>(ta + oA);
        xa[k][1] = *reinterpret_cast<const uint4*>(ta + oB);
        if (tb != nullptr) {
          xb[k][0] = *reinterpret_cast<const uint4*>(tb + oA);
          xb[k][1] = *reinterpret_cast<const uint4*>(tb + oB);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < NB; ++k) {
      if (!live[k]) continue;
      const int task = base + k * nthreads;
      const int r = task >> 3, au = task & 7, a = au >> 1, u = au & 1, hi = a >> 1;
      // s' = -s for the first block's items (sin is the high half of a word)
      const uint32_t flip = hi ? 0u : 0x80000000u;
      const uint32_t ww[8] = {w[k][0].x ^ flip, w[k][0].y ^ flip, w[k][0].z ^ flip,
                              w[k][0].w ^ flip, w[k][1].x ^ flip, w[k][1].y ^ flip,
                              w[k][1].z ^ flip, w[k][1].w ^ flip};
      uint64_t c2[4], s2[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        c2[q] = f2_pack(bf16_lo(ww[2 * q]), bf16_lo(ww[2 * q + 1]));
        s2[q] = f2_pack(bf16_hi(ww[2 * q]), bf16_hi(ww[2 * q + 1]));
      }
      const int c1 = 4 * (a & 1) + u;
      const uint32_t oA = hi * kBlkBytes + sw128_offset(r, hi ? c1 + 2 : c1);
      const uint32_t oB = hi * kBlkBytes + sw128_offset(r, hi ? c1 : c1 + 2);
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (m == 1 && tb == nullptr) break;
        uint8_t* t = m ? tb : ta;
        const uint4 vA = m ? xb[k][0] : xa[k][0], vB = m ? xb[k][1] : xa[k][1];
        const uint32_t xA[4] = {vA.x, vA.y, vA.z, vA.w};
        const uint32_t xB[4] = {vB.x, vB.y, vB.z, vB.w};
        uint32_t yA[4], yB[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint64_t a2 = f2_pack(bf16_lo(xA[q]), bf16_hi(xA[q]));
          const uint64_t b2 = f2_pack(bf16_lo(xB[q]), bf16_hi(xB[q]));
          float y0, y1, z0, z1;
          f2_unpack(fadd2(fmul2(a2, c2[q]), fmul2(b2, s2[q])), y0, y1);
          f2_unpack(fsub2(fmul2(b2, c2[q]), fmul2(a2, s2[q])), z0, z1);
          yA[q] = pack_bf16(y0, y1);
          yB[q] = pack_bf16(z0, z1);
        }
        *reinterpret_cast<uint4*>(t + oA) = make_uint4(yA[0], yA[1], yA[2], yA[3]);
        *reinterpret_cast<uint4*>(t + oB) = make_uint4(yB[0], yB[1], yB[2], yB[3]);
      }
    }
  }
}

// K/V tile visited at step j by the CTA with tile pair `pair`.
__device__ __forceinline__ int kv_tile_of(int j, int pair, int nkv) {
  const int t = j + (2 * pair) % nkv;
  return t >= nkv ? t - nkv : t;
}

struct Params {
  int S, H, kv_len, nkv;
  float scale_log2;  // scale * log2(e)
  float* lse;        // (B, H, S)
  // Sequence-block folding (ring attention): 0 plain (O through tm_o, LSE);
  // 1 first block: (o_acc, lse_acc) <- this block; 2 fold this block into
  // (o_acc, lse_acc); 3 fold, then write the final O (tm_o) and LSE (lse).
  int merge;
  float* o_acc;      // fp32 contiguous (B, S, H, D), normalised rows
  float* lse_acc;    // (B, H, S), natural log
  // RoPE inside (plain mode, kv_len == S): packed bf16 (cos, sin) per
  // (token, frequency), 64 words per token; nullptr: q, k used as given
  const uint32_t* rope_cs;
  // per (b, h, K tile): set once the tile's rotated copy is in k_rot
  uint32_t* k_pub;
};

__global__ void __launch_bounds__(kThreads, 1)
attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q,
                const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v,
                const __grid_constant__ CUtensorMap tm_o,
                const __grid_constant__ CUtensorMap tm_qr,
                const __grid_constant__ CUtensorMap tm_kr, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kOffBar);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile int* abort_flag =
      reinterpret_cast<volatile int*>(smem + kOffMisc + 4);
  // per ring slot, with RoPE inside: 1 = the K tile in the slot is raw and
  // is rotated here, 0 = it is another CTA's published rotated copy
  volatile int* rot_mark = reinterpret_cast<volatile int*>(smem + kOffMisc + 16);

  const int warp = warp_id();
  const int lane = lane_id();
  const int pair = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int nkv = p.nkv;

  if (threadIdx.x == 0) {
    mbar_init(&bars[B_Q], 1);
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&bars[B_FULL + s], 1);
      mbar_init(&bars[B_KFULL + s], 1);
      mbar_init(&bars[B_EMPTY + s], 1);
    }
    for (int t = 0; t < kTiles; ++t) {
      mbar_init(&bars[B_SFULL + t], 1);
      mbar_init(&bars[B_PREADY + t], 128);
      mbar_init(&bars[B_PVDONE + t], 1);
    }
    mbar_init(&bars[B_FINAL], 1);
    for (int s = 0; s < kSlots; ++s) mbar_init(&bars[B_KREADY + s], 64);
    mbar_init(&bars[B_QREADY], 256);
    mbar_init(&bars[B_STORED], 2);
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
    // ------------------------------------------------ producer: Q0, Q1, K, V
    if (lane == 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      if (p.rope_cs != nullptr) {
        // this CTA's own K tiles (steps 0 and 1) are being rotated here: a
        // CTA that needs them waits for their publication instead of rotating
        uint32_t* pub = p.k_pub + ((int64_t)b * p.H + h) * nkv;
        atom_max_relaxed_gpu(pub + kv_tile_of(0, pair, nkv), 1u);
        if (nkv > 1) atom_max_relaxed_gpu(pub + kv_tile_of(1, pair, nkv), 1u);
      }
      const int row = pair * kTiles * kRows;
      mbar_arrive_expect_tx(&bars[B_Q], kTiles * kTileBytes);
      for (int t = 0; t < kTiles; ++t) {
        uint8_t* d = smem + kOffQ + t * kTileBytes;
        tma_load_4d(d, &tm_q, &bars[B_Q], 0, row + t * kRows, h, b);
        tma_load_4d(d + kBlkBytes, &tm_q, &bars[B_Q], 64, row + t * kRows, h, b);
      }
      bool ok = true;
      for (int n = 0; n < 2 * nkv; ++n) {
        if (*abort_flag) break;
        const int s = n % kSlots, u = n / kSlots;
        if (n >= kSlots && !(ok = mbar_wait(&bars[B_EMPTY + s], (u - 1) & 1))) break;
        // the slots of the first two K tiles are stored to k_rot from shared
        // memory: their first reuse waits until those stores have read them
        if (p.rope_cs != nullptr && n == kSlots && !(ok = mbar_wait(&bars[B_STORED], 0))) break;
        uint8_t* d = smem + kOffKV + s * kTileBytes;
        const int kvt = kv_tile_of(n >> 1, pair, nkv);
        const CUtensorMap* tm = (n & 1) ? &tm_v : &tm_k;
        if (!(n & 1) && p.rope_cs != nullptr) {
          // a K tile other than this CTA's own two: its rotated copy when
          // the CTA that owns it has published it (checked, never waited for)
          bool published = false;
          if ((n >> 1) >= 2) {
            const uint32_t* flag = p.k_pub + ((int64_t)b * p.H + h) * nkv + kvt;
            uint32_t state = ld_acquire_gpu(flag);
            if (state == 1u) {  // the owner runs: it publishes within a step or two
              const long long t0 = clock64();
              while ((state = ld_acquire_gpu(flag)) == 1u && clock64() - t0 < kPubWaitCycles &&
                     !*abort_flag)
                __nanosleep(128);
            }
            published = state == 2u;
            if (published) fence_proxy_async_global();
          }
          rot_mark[s] = published ? 0 : 1;
          if (published) tm = &tm_kr;
        }
        uint64_t* full = &bars[((n & 1) ? B_FULL : B_KFULL) + s];
        mbar_arrive_expect_tx(full, kTileBytes);
        const int kvrow = kvt * kKeys;
        tma_load_4d(d, tm, full, 0, kvrow, h, b);
        tma_load_4d(d + kBlkBytes, tm, full, 64, kvrow, h, b);
      }
      if (!ok) *abort_flag = 1;
    }
  } else if (warp == 9) {
    // ---------------------------------------- MMA issuer (whole warp, one lane issues)
    {
      constexpr uint32_t kIdescS = idesc_bf16(128, 128, false, false);
      constexpr uint32_t kIdescO = idesc_bf16(128, 128, false, true);
      const bool rotate = p.rope_cs != nullptr;
      bool ok = mbar_wait_w(&bars[B_Q], 0);  // (with RoPE: QREADY, waited in issue_s)
      tc_fence_after();
      // S_t(j) = Q_t K_j^T. It overwrites P_t(j-1), which PV_t(j-1) reads:
      // tcgen05.mma operations issued by one thread execute in issue order,
      // so S_t(j) is issued right behind PV_t(j-1) without waiting for it.
      // With RoPE inside, K_j is used once rotated (KREADY of its slot: the
      // slot holds K tiles at steps j, j+5, ..., so that barrier's phase is
      // j / 5) and Q_t once its warpgroup has rotated it (QREADY).
      auto issue_s = [&](int t, int j) -> bool {
        const int s = (2 * j) % kSlots;
        if (t == 0) {
          // RoPE inside: steps 0, 1 use the tiles the softmax warpgroups
          // rotated (QREADY); a slot holds a later K tile at steps j, j+5,
          // ..., so its KREADY phase is (j - 2) / 5
          if (rotate ? (j < 2 ? (j == 0 && !mbar_wait_w(&bars[B_QREADY], 0))
                              : !mbar_wait_w(&bars[B_KREADY + s], ((j - 2) / kSlots) & 1))
                     : !mbar_wait_w(&bars[B_KFULL + s], (2 * j / 10) & 1))
            return false;
        }
        tc_fence_after();
        const uint32_t q_base = smem_u32(smem + kOffQ + t * kTileBytes);
        const uint32_t k_base = smem_u32(smem + kOffKV + s * kTileBytes);
        const uint32_t d = tmem + kColS + (uint32_t)t * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ss_w(d, kmajor_desc(q_base, kk, kBlkBytes),
                    kmajor_desc(k_base, kk, kBlkBytes), kIdescS, kk > 0);
        umma_commit_w(&bars[B_SFULL + t]);
        if (t == kTiles - 1) umma_commit_w(&bars[B_EMPTY + s]);
        return true;
      };
      // O_t += P_t(j) V_j
      auto issue_pv = [&](int t, int j) -> bool {
        const int s = (2 * j + 1) % kSlots;
        if (t == 0 && !mbar_wait_w(&bars[B_FULL + s], ((2 * j + 1) / 10) & 1)) return false;
        if (!mbar_wait_w(&bars[B_PREADY + t], j & 1)) return false;
        tc_fence_after();
        const uint32_t v_base = smem_u32(smem + kOffKV + s * kTileBytes);
        const uint32_t p_col = tmem + kColS + (uint32_t)t * 128u;
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_ts_w(tmem + kColO + (uint32_t)t * 128u, p_col + kk * 8,
                    mnmajor_desc(v_base, kk, kBlkBytes), kIdescO,
                    (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit_w(&bars[B_PVDONE + t]);
        if (t == kTiles - 1) umma_commit_w(&bars[B_EMPTY + s]);
        return true;
      };
      if (ok) ok = issue_s(0, 0);
      if (ok) ok = issue_s(1, 0);
      for (int j = 0; ok && j < nkv; ++j) {
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
        for (int t = 0; ok && t < kTiles; ++t) {
          ok = issue_pv(t, j);
          if (ok && j + 1 < nkv) ok = issue_s(t, j + 1);
        }
      }
      if (!ok && lane == 0) *abort_flag = 1;
      // drain: every MMA issued above completes before TMEM is released
      umma_commit_w(&bars[B_FINAL]);
      mbar_wait(&bars[B_FINAL], 0);
    }
  } else if (warp < 8) {
    // ------------------------------------------------------------- softmax
    const int t = warp >> 2;                  // Q tile of this warpgroup
    const int sub = warp & 3;                 // TMEM lane quarter
    const int row_in_tile = sub * 32 + lane;
    const uint32_t lane_off = (uint32_t)(sub * 32) << 16;
    const uint32_t t_s = tmem + lane_off + kColS + (uint32_t)t * 128u;
    const uint32_t t_o = tmem + lane_off + kColO + (uint32_t)t * 128u;
    const int bar_id = 1 + t;                 // named barrier of the warpgroup
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;
    float l_run = 0.f;
    bool failed = false;
    const bool own_k = p.rope_cs != nullptr && t < nkv;  // this warpgroup rotates own K tile t
    if (p.rope_cs != nullptr) {
      // RoPE inside: rotate Q tile t and this CTA's own K tile t (the K tile
      // of step t, in ring slot 2t) in place, store both to q_rot / k_rot
      uint8_t* qt = smem + kOffQ + t * kTileBytes;
      uint8_t* kt = smem + kOffKV + 2 * t * kTileBytes;
      const int q_row0 = (pair * kTiles + t) * kRows;
      const int k_row0 = kv_tile_of(t, pair, nkv) * kKeys;
      bool stop = !mbar_wait(&bars[B_Q], 0);
      if (!stop && own_k) stop = !mbar_wait(&bars[B_KFULL + 2 * t], 0);
      stop = __any_sync(0xffffffffu, stop);
      if (!stop) {
        if (own_k && k_row0 == q_row0) {  // (kv_len == S: the same tokens and limit)
          rope_rotate_rows<4>(qt, kt, p.rope_cs, q_row0, p.S, row_in_tile, 128);
        } else {
          rope_rotate_rows<8>(qt, nullptr, p.rope_cs, q_row0, p.S, row_in_tile, 128);
          if (own_k) rope_rotate_rows<8>(kt, nullptr, p.rope_cs, k_row0, p.kv_len, row_in_tile, 128);
        }
      }
      fence_proxy_async_smem();
      if (named_bar_any(bar_id, 128, stop)) {
        failed = true;
      } else if (warp == 4 * t && lane == 0) {
        tma_store_4d(&tm_qr, qt, 0, q_row0, h, b);
        tma_store_4d(&tm_qr, qt + kBlkBytes, 64, q_row0, h, b);
        if (own_k) {
          tma_store_4d(&tm_kr, kt, 0, k_row0, h, b);
          tma_store_4d(&tm_kr, kt + kBlkBytes, 64, k_row0, h, b);
        }
        bulk_commit_group();
      }
      mbar_arrive(&bars[B_QREADY]);
      if (warp == 4 * t && lane == 0) {
        // the producer reuses the K slots only once these stores have read them
        bulk_wait_group_read0();
        mbar_arrive(&bars[B_STORED]);
      }
    }
    for (int j = 0; j < nkv; ++j) {
      if (j == 1 && own_k && warp == 4 * t && lane == 0 && !failed) {
        // a step later the K store has completed (no wait in practice):
        // publish the tile (a proxy fence orders the TMA writes before the
        // release of the flag)
        bulk_wait_group0();
        fence_proxy_async_global();
        st_release_gpu(p.k_pub + ((int64_t)b * p.H + h) * nkv + kv_tile_of(t, pair, nkv), 2u);
      }
      bool stop = failed || *abort_flag != 0;
      if (!stop) stop = !mbar_wait(&bars[B_SFULL + t], j & 1);
      if (__any_sync(0xffffffffu, stop)) { failed = true; break; }
      tc_fence_after();
      uint32_t sr[128];
      tmem_ld32(t_s + 0, sr);
      tmem_ld32(t_s + 32, sr + 32);
      tmem_ld32(t_s + 64, sr + 64);
      tmem_ld32(t_s + 96, sr + 96);
      tmem_wait_ld();
      float* sv = reinterpret_cast<float*>(sr);
      const int valid = p.kv_len - kv_tile_of(j, pair, nkv) * kKeys;
      if (valid < kKeys) {
#pragma unroll
        for (int c = 0; c < kKeys; ++c)
          if (c >= valid) sv[c] = -INFINITY;
      }
      // row maximum: four independent chains of three-input maxima
      float m4[4] = {sv[0], sv[1], sv[2], sv[3]};
#pragma unroll
      for (int c = 4; c < kKeys; c += 8) {
#pragma unroll
        for (int k = 0; k < 4; ++k) m4[k] = fmax3(m4[k], sv[c + 2 * k], sv[c + 2 * k + 1]);
      }
      const float mx = fmax3(fmaxf(m4[0], m4[1]), m4[2], m4[3]);
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
      // P = 2^(S*scale*log2e - m): packed bf16 pairs written over the
      // registers already consumed; four partial sums
      // (pairs of columns through the packed fp32x2 FMA / add)
      const uint64_t sl2_2 = f2_pack(sl2, sl2), negm_2 = f2_pack(-m_use, -m_use);
      uint64_t sum2[2] = {0ull, 0ull};
#pragma unroll
      for (int i = 0; i < kKeys / 2; ++i) {
        float x0, x1;
        f2_unpack(ffma2(f2_pack(sv[2 * i], sv[2 * i + 1]), sl2_2, negm_2), x0, x1);
        const float p0 = poly_column(2 * i) ? exp2_poly(x0) : fast_exp2(x0);
        const float p1 = poly_column(2 * i + 1) ? exp2_poly(x1) : fast_exp2(x1);
        sum2[i & 1] = fadd2(sum2[i & 1], f2_pack(p0, p1));
        sr[i] = pack_bf16(p0, p1);
      }
      float sum4[4];
      f2_unpack(sum2[0], sum4[0], sum4[1]);
      f2_unpack(sum2[1], sum4[2], sum4[3]);
      tmem_st32(t_s + 0, sr);
      tmem_st32(t_s + 32, sr + 32);
      // O_t may only be rescaled while no PV_t is in flight: after PV_t(j-1)
      // (already complete: S_t(j) was issued after it)
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.f)) {
        if (!__all_sync(0xffffffffu, mbar_wait(&bars[B_PVDONE + t], (j - 1) & 1))) {
          failed = true;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int cb = 0; cb < 8; ++cb) {
          uint32_t orow[16];
          tmem_ld16(t_o + cb * 16, orow);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 16; ++i)
            orow[i] = __float_as_uint(__uint_as_float(orow[i]) * alpha);
          tmem_st16(t_o + cb * 16, orow);
        }
      }
      tmem_wait_st();
      l_run = l_run * alpha + ((sum4[0] + sum4[1]) + (sum4[2] + sum4[3]));
      m_run = m_use;
      tc_fence_before();
      mbar_arrive(&bars[B_PREADY + t]);
    }
    // epilogue: O_t / l to bf16, staged in the Q_t tile (free: every S_t MMA
    // completed before the last PV_t), stored with two TMA tile stores
    bool stop = failed || *abort_flag != 0;
    if (!stop) stop = !mbar_wait(&bars[B_PVDONE + t], (nkv - 1) & 1);
    stop = __any_sync(0xffffffffu, stop);
    // (the rotation flag is re-read from the parameters: no register held
    // across the loop)
    if (p.rope_cs != nullptr && warp == 4 * t && lane == 0) bulk_wait_group_read0();
    if (!named_bar_any(bar_id, 128, stop)) {
      tc_fence_after();
      const int row0 = (pair * kTiles + t) * kRows;
      const int row = row0 + row_in_tile;
      const bool live = row < p.S;
      const float lse_blk = (m_run + __log2f(l_run)) * 0.69314718055994531f;
      // this row's O = wb * (block O / l) + wa * o_acc, LSE = lse_out
      float wb = 1.f / l_run, wa = 0.f, lse_out = lse_blk;
      const int64_t acc_row = (((int64_t)b * p.S + row) * p.H + h) * 128;
      if (p.merge >= 2 && live) {
        const float la = p.lse_acc[((int64_t)b * p.H + h) * p.S + row];
        const float mx = fmaxf(la, lse_blk);
        const float ea = expf(la - mx), eb = expf(lse_blk - mx);
        const float inv = 1.f / (ea + eb);
        wa = ea * inv;
        wb = eb * inv / l_run;
        lse_out = mx + logf(ea + eb);
      }
      uint8_t* stage = smem + kOffQ + t * kTileBytes;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t orow[64];
        tmem_ld32(t_o + half * 64, orow);
        tmem_ld32(t_o + half * 64 + 32, orow + 32);
        tmem_wait_ld();
        float* ov = reinterpret_cast<float*>(orow);
#pragma unroll
        for (int c = 0; c < 64; ++c) ov[c] *= wb;
        if (p.merge >= 2 && live) {
          const float4* a4 = reinterpret_cast<const float4*>(p.o_acc + acc_row + half * 64);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const float4 a = a4[c];
            ov[4 * c + 0] = fmaf(a.x, wa, ov[4 * c + 0]);
            ov[4 * c + 1] = fmaf(a.y, wa, ov[4 * c + 1]);
            ov[4 * c + 2] = fmaf(a.z, wa, ov[4 * c + 2]);
            ov[4 * c + 3] = fmaf(a.w, wa, ov[4 * c + 3]);
          }
        }
        if (p.merge == 1 || p.merge == 2) {
          if (live) {
            float4* d4 = reinterpret_cast<float4*>(p.o_acc + acc_row + half * 64);
#pragma unroll
            for (int c = 0; c < 16; ++c)
              d4[c] = make_float4(ov[4 * c], ov[4 * c + 1], ov[4 * c + 2], ov[4 * c + 3]);
          }
        } else {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint4 v;
            v.x = pack_bf16(ov[c * 8 + 0], ov[c * 8 + 1]);
            v.y = pack_bf16(ov[c * 8 + 2], ov[c * 8 + 3]);
            v.z = pack_bf16(ov[c * 8 + 4], ov[c * 8 + 5]);
            v.w = pack_bf16(ov[c * 8 + 6], ov[c * 8 + 7]);
            *reinterpret_cast<uint4*>(stage + half * kBlkBytes + sw128_offset(row_in_tile, c)) = v;
          }
        }
      }
      if (p.merge == 0 || p.merge == 3) {
        fence_proxy_async_smem();
        named_bar_sync(bar_id, 128);
        if (warp == 4 * t && lane == 0) {
          tma_store_4d(&tm_o, stage, 0, row0, h, b);
          tma_store_4d(&tm_o, stage + kBlkBytes, 64, row0, h, b);
          bulk_commit_group();
          bulk_wait_group0();
        }
      }
      if (live) {
        const int64_t li = ((int64_t)b * p.H + h) * p.S + row;
        if (p.merge == 1 || p.merge == 2) p.lse_acc[li] = lse_out;
        else p.lse[li] = lse_out;
      }
    } else {
      *abort_flag = 1;
    }
    if (p.rope_cs != nullptr && warp == 4 * t && lane == 0) bulk_wait_group0();
  } else if (warp >= 10) {
    // ---------- RoPE inside: rotate the K tiles of steps >= 2 that arrived
    // unrotated (their owner had not published them in time)
    if (p.rope_cs != nullptr) {
      const int tid = threadIdx.x - 320;  // 0..63
      bool ok = true;
      // every K tile's arrival is waited for in order (also those of steps
      // 0 and 1, which the softmax warpgroups rotate), so no phase of a K
      // barrier is ever skipped
      for (int j = 0; j < nkv; ++j) {
        const int n = 2 * j, s = n % kSlots;
        if (__any_sync(0xffffffffu, *abort_flag != 0)) { ok = false; break; }
        if (!(ok = mbar_wait_w(&bars[B_KFULL + s], (n / 10) & 1))) break;
        if (j < 2) continue;
        if (rot_mark[s]) {
          rope_rotate_rows<8>(smem + kOffKV + s * kTileBytes, nullptr, p.rope_cs,
                              kv_tile_of(j, pair, nkv) * kKeys, p.kv_len, tid, 64);
          fence_proxy_async_smem();
        }
        mbar_arrive(&bars[B_KREADY + s]);
      }
      if (!ok) *abort_flag = 1;
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
                         cudaStream_t stream, int merge, float* o_acc,
                         float* lse_acc, const FwdRope* rope) {
  if (rope != nullptr &&
      (merge != 0 || kv_len != sh.S || rope->cs == nullptr || rope->k_pub == nullptr))
    return FA_ERR_INVALID_ARG;  // in-tile rotation: plain mode, q and k share positions
  CUtensorMap tq, tk, tv, to, tqr, tkr;
  int rc = make_tmap_bshd(&tq, q, sh.B, sh.S, sh.H, sh.D, 128);
  if (!rc) rc = make_tmap_bshd(&tk, k, sh.B, kv_len, sh.H, sh.D, 128);
  if (!rc) rc = make_tmap_bshd(&tv, v, sh.B, kv_len, sh.H, sh.D, 128);
  // modes 1 and 2 write no bf16 O: the map is encoded over q and never used
  if (!rc) rc = make_tmap_bshd(&to, (merge == 1 || merge == 2) ? q : o, sh.B, sh.S, sh.H, sh.D, 128);
  // the rotated-q/k maps exist only with RoPE inside (else never used)
  if (!rc) rc = make_tmap_bshd(&tqr, rope ? rope->q_rot : q, sh.B, sh.S, sh.H, sh.D, 128);
  if (!rc) rc = make_tmap_bshd(&tkr, rope ? rope->k_rot : q, sh.B, sh.S, sh.H, sh.D, 128);
  if (rc) return rc;
  fwd::Params p;
  p.S = sh.S;
  p.H = sh.H;
  p.kv_len = kv_len;
  p.nkv = (kv_len + fwd::kKeys - 1) / fwd::kKeys;
  p.scale_log2 = scale * 1.4426950408889634f;
  p.lse = lse;
  p.merge = merge;
  p.o_acc = o_acc;
  p.lse_acc = lse_acc;
  p.rope_cs = rope ? rope->cs : nullptr;
  p.k_pub = rope ? rope->k_pub : nullptr;
  rc = ensure_smem_attr((const void*)fwd::attn_fwd_kernel, fwd::kSmemBytes,
                        kKernelFwdBf16);
  if (rc) return rc;
  constexpr int kRowsPerCta = fwd::kTiles * fwd::kRows;
  dim3 grid((sh.S + kRowsPerCta - 1) / kRowsPerCta, sh.H, sh.B);
  fwd::attn_fwd_kernel<<<grid, fwd::kThreads, fwd::kSmemBytes, stream>>>(
      tq, tk, tv, to, tqr, tkr, p);
  return launch_status();
}

int fwd_device_status() { return tu_device_status(); }

}  // namespace fa
