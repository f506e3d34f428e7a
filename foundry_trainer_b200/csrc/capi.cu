// capi.cu — the extern "C" entry points of include/foundry_attn.h:
// argument validation, workspace carving, and the launch sequences of the
// forward, backward and sequence-shard building blocks.
#include <cudaTypedefs.h>

#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <utility>
#include <vector>

#include "attn_common.h"
#include "rope.cuh"
#include "sm100_ptx.cuh"

namespace fa {


// ------------------------------------------------------------ TMA encoding
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

static int encode_bshd(CUtensorMap* map, const fa_tensor_t* t, int B, int S,
                       int H, int D, int box_rows, CUtensorMapDataType dt,
                       int esize, int box_inner) {
  auto enc = encode_fn();
  if (!enc) return FA_ERR_LAUNCH;
  if (t->stride_d != 1) return FA_ERR_ALIGNMENT;
  // Size-1 modes may carry any stride; give them a legal one.
  int64_t ss = t->stride_s, sh = t->stride_h, sb = t->stride_b;
  if (H == 1) sh = (int64_t)D;
  if (S == 1) ss = (int64_t)D * H;
  if (B == 1) sb = (int64_t)S * ss;
  cuuint64_t dims[4] = {(cuuint64_t)D, (cuuint64_t)S, (cuuint64_t)H, (cuuint64_t)B};
  cuuint64_t strides[3] = {(cuuint64_t)(ss * esize), (cuuint64_t)(sh * esize),
                           (cuuint64_t)(sb * esize)};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 != 0 || strides[i] >= (1ull << 40)) return FA_ERR_ALIGNMENT;
  if (reinterpret_cast<uintptr_t>(t->data) % 16 != 0) return FA_ERR_ALIGNMENT;
  cuuint32_t box[4] = {(cuuint32_t)box_inner, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dt, 4, t->data, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FA_OK : FA_ERR_ALIGNMENT;
}

int make_tmap_bshd(CUtensorMap* map, const fa_tensor_t* t, int B, int S, int H,
                   int D, int box_rows) {
  return encode_bshd(map, t, B, S, H, D, box_rows,
                     CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, 64);
}

int make_tmap_bshd_f32(CUtensorMap* map, const fa_tensor_t* t, int B, int S,
                       int H, int D, int box_rows) {
  return encode_bshd(map, t, B, S, H, D, box_rows,
                     CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, 32);
}

// ------------------------------------------------------ CUDA error text
static thread_local char g_last_error[256] = "";

int record_cuda_error(cudaError_t e) {
  if (e == cudaSuccess) return FA_OK;
  std::snprintf(g_last_error, sizeof(g_last_error), "%s: %s", cudaGetErrorName(e),
                cudaGetErrorString(e));
  return FA_ERR_LAUNCH;
}

int launch_status() { return record_cuda_error(cudaGetLastError()); }

void record_error_text(const char* msg) {
  std::snprintf(g_last_error, sizeof(g_last_error), "%s", msg);
}

// ------------------------------------------------- per-device attributes
static std::atomic<int> g_attr_done[64][kKernelCount];

int ensure_smem_attr(const void* fn, int bytes, int kernel_id) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return FA_ERR_NO_DEVICE;
  if (g_attr_done[dev][kernel_id].load(std::memory_order_acquire)) return FA_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return record_cuda_error(e);
  g_attr_done[dev][kernel_id].store(1, std::memory_order_release);
  return FA_OK;
}

RopeArgs make_rope_args(const fa_rope_t* rope, int round_bf16, int pos_offset) {
  RopeArgs r;
  std::memset(&r, 0, sizeof(r));
  if (rope == nullptr) return r;
  r.pos = rope->pos;
  r.n_axes = rope->n_axes;
  r.axis_dim = rope->axis_dim;
  r.round_bf16 = round_bf16;
  r.pos_offset = pos_offset;
  const int half = rope->axis_dim / 2;
  for (int a = 0; a < rope->n_axes; ++a)
    for (int j = 0; j < half; ++j)
      r.inv_freq[a * half + j] = (float)std::pow(
          (double)rope->theta, -2.0 * (double)j / (double)rope->axis_dim);
  return r;
}

// --------------------------------------------------------------- validation
static int check_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return FA_ERR_NO_DEVICE;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) !=
      cudaSuccess)
    return FA_ERR_NO_DEVICE;
  return major == 10 ? FA_OK : FA_ERR_NO_DEVICE;
}

static int check_tensor(const fa_tensor_t* t, int esize, bool tma) {
  if (t == nullptr || t->data == nullptr) return FA_ERR_INVALID_ARG;
  if (t->stride_d != 1) return FA_ERR_ALIGNMENT;
  if (tma) {
    if (reinterpret_cast<uintptr_t>(t->data) % 16 != 0) return FA_ERR_ALIGNMENT;
  } else if (reinterpret_cast<uintptr_t>(t->data) % esize != 0) {
    return FA_ERR_ALIGNMENT;
  }
  return FA_OK;
}

int check_attn_shape(int dtype, int B, int S, int H, int D) {
  if (dtype != FA_DTYPE_F32 && dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (B <= 0 || S <= 0 || H <= 0 || D <= 0) return FA_ERR_INVALID_ARG;
  if (D != 128) return FA_ERR_UNSUPPORTED;
  if ((int64_t)B * S * H * D >= (int64_t)1 << 40) return FA_ERR_TOO_LARGE;
  if (B > 65535 || H > 65535) return FA_ERR_TOO_LARGE;
  return FA_OK;
}

static int check_rope(const fa_rope_t* rope, int D) {
  if (rope == nullptr) return FA_OK;
  if (rope->pos == nullptr) return FA_ERR_INVALID_ARG;
  if (rope->n_axes <= 0 || rope->axis_dim <= 0 || (rope->axis_dim & 1))
    return FA_ERR_UNSUPPORTED;
  if (rope->n_axes * rope->axis_dim != D) return FA_ERR_UNSUPPORTED;
  if (rope->n_axes * rope->axis_dim / 2 > kMaxRopeFreqs) return FA_ERR_UNSUPPORTED;
  if (!(rope->theta > 0.f)) return FA_ERR_INVALID_ARG;
  return FA_OK;
}

static size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

// bytes of the per-call (cos, sin) table: S tokens x n_axes*axis_dim/2 float2
static size_t rope_table_bytes(int S, const fa_rope_t* rope) {
  if (rope == nullptr) return 0;
  return align256((size_t)S * (size_t)(rope->n_axes * (rope->axis_dim / 2)) * sizeof(float2));
}

static fa_tensor_t contiguous_view(void* p, int S, int H, int D) {
  fa_tensor_t t;
  t.data = p;
  t.stride_d = 1;
  t.stride_h = D;
  t.stride_s = (int64_t)H * D;
  t.stride_b = (int64_t)S * H * D;
  return t;
}

// ------------------------------------------- per-kernel CUDA-event timing
// Optional measurement hook: when enabled, the main forward / backward kernel
// launches are bracketed by CUDA events on their own stream so a benchmark can
// read each kernel's device time without a profiler. One device per process.
struct TimerSlot {
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pairs;
  size_t used = 0;
};
static std::mutex g_timer_mu;
static std::atomic<int> g_timing{0};
static TimerSlot g_slots[FA_TIMER_COUNT];

static cudaEvent_t timer_begin(int id, cudaStream_t st) {
  if (!g_timing.load(std::memory_order_relaxed)) return nullptr;
  std::lock_guard<std::mutex> lk(g_timer_mu);
  TimerSlot& s = g_slots[id];
  if (s.used == s.pairs.size()) {
    cudaEvent_t a, b;
    if (cudaEventCreate(&a) != cudaSuccess) return nullptr;
    if (cudaEventCreate(&b) != cudaSuccess) {
      cudaEventDestroy(a);
      return nullptr;
    }
    s.pairs.emplace_back(a, b);
  }
  auto& pr = s.pairs[s.used++];
  cudaEventRecord(pr.first, st);
  return pr.second;
}

static void timer_end(cudaEvent_t stop, cudaStream_t st) {
  if (stop != nullptr) cudaEventRecord(stop, st);
}

#define FA_TRY(expr)            \
  do {                          \
    int _rc = (expr);           \
    if (_rc != FA_OK) return _rc; \
  } while (0)

}  // namespace fa

using namespace fa;

extern "C" {

const char* fa_status_string(int status) {
  switch (status) {
    case FA_OK: return "ok";
    case FA_ERR_INVALID_ARG: return "invalid argument";
    case FA_ERR_UNSUPPORTED: return "unsupported dtype, head_dim or rope layout";
    case FA_ERR_ALIGNMENT: return "stride or pointer violates TMA alignment (16 B)";
    case FA_ERR_LAUNCH: return "CUDA launch or runtime call failed";
    case FA_ERR_DEVICE_TIMEOUT: return "device-side bounded wait expired";
    case FA_ERR_WORKSPACE: return "workspace missing or too small";
    case FA_ERR_NO_DEVICE: return "no sm_100 device current";
    case FA_ERR_TOO_LARGE: return "size beyond addressing limits";
    default: return "unknown status";
  }
}

int fa_abi_version(void) { return FA_ABI_VERSION; }

const char* fa_last_error(void) { return g_last_error; }

const char* fa_build_info(void) {
  return "foundry_attn sm_100a (tcgen05/TMEM/TMA bf16 path, fp32 SIMT path)";
}

int fa_device_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return FA_ERR_LAUNCH;
  // every translation unit's word is read (and cleared); the first code wins
  int first = 0;
  for (int v : {fwd_device_status(), bwd_device_status(), f32_device_status(),
                misc_device_status(), qkp_device_status(), peer_device_status()}) {
    if (v < 0) return FA_ERR_LAUNCH;
    if (first == 0) first = v;
  }
  return first;
}

// bf16 forward with the reference's rope layout (four 32-wide axes): the
// rotation runs inside the forward kernel's tile loads
static bool fused_fwd_rope(int dtype, const fa_rope_t* rope, int D) {
  return dtype == FA_DTYPE_BF16 && rope != nullptr && D == 128 && rope->n_axes == 4 &&
         rope->axis_dim == 32;
}

// forward workspace (RoPE inside the op): [q_rot | k_rot | (cos, sin) table
// (float2) | the same as packed bf16 pairs (in-kernel rotation only)]
size_t fa_fwd_workspace_bytes(int dtype, int B, int S, int H, int D,
                              const fa_rope_t* rope) {
  if (rope == nullptr) return 0;
  const size_t es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  size_t total = 2 * align256((size_t)B * S * H * D * es) + rope_table_bytes(S, rope);
  if (fused_fwd_rope(dtype, rope, D))  // + packed table + per-K-tile publish flags
    total += rope_table_bytes(S, rope) / 2 + align256((size_t)B * H * ((S + 127) / 128) * 4);
  return total;
}

int fa_fwd(int dtype, int B, int S, int H, int D, const fa_tensor_t* q,
           const fa_tensor_t* k, const fa_tensor_t* v, const fa_tensor_t* o,
           float* lse, float scale, const fa_rope_t* rope, void* workspace,
           size_t workspace_bytes, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  FA_TRY(check_rope(rope, D));
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  const bool bf = dtype == FA_DTYPE_BF16;
  const int es = bf ? 2 : 4;
  FA_TRY(check_tensor(q, es, bf));
  FA_TRY(check_tensor(k, es, bf));
  FA_TRY(check_tensor(v, es, bf));
  FA_TRY(check_tensor(o, es, true));
  if (lse == nullptr) return FA_ERR_INVALID_ARG;
  FA_TRY(check_sm100());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const AttnShape sh{B, S, H, D};
  fa_tensor_t qr = *q, kr = *k;
  if (rope != nullptr) {
    const size_t need = fa_fwd_workspace_bytes(dtype, B, S, H, D, rope);
    if (workspace == nullptr || workspace_bytes < need) return FA_ERR_WORKSPACE;
    uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
    const size_t tb = align256((size_t)B * S * H * D * es);
    qr = contiguous_view(ws, S, H, D);
    kr = contiguous_view(ws + tb, S, H, D);
    float2* table = reinterpret_cast<float2*>(ws + 2 * tb);
    if (fused_fwd_rope(dtype, rope, D)) {
      // the kernel rotates q and k in its tile loads and writes q_rot and
      // k_rot; the table pass also leaves the float2 table for fa_bwd_saved
      uint32_t* packed = reinterpret_cast<uint32_t*>(ws + 2 * tb + rope_table_bytes(S, rope));
      uint32_t* k_pub = packed + rope_table_bytes(S, rope) / 8;
      const int64_t n_pub = (int64_t)B * H * ((S + 127) / 128);
      FA_TRY(launch_rope_table2(S, rope, table, packed, k_pub, n_pub, st));
      const FwdRope fr{packed, &qr, &kr, k_pub};
      cudaEvent_t stop = timer_begin(FA_TIMER_FWD, st);
      const int rc = launch_attn_fwd_bf16(sh, S, q, k, v, o, lse, scale, st, 0, nullptr,
                                          nullptr, &fr);
      timer_end(stop, st);
      return rc;
    }
    // the rotation pass also leaves the (cos, sin) table for fa_bwd_saved
    FA_TRY(launch_rope_pair(dtype, sh, q, &qr, k, &kr, rope, 0, 0, st, nullptr, table));
  }
  cudaEvent_t stop = timer_begin(FA_TIMER_FWD, st);
  const int rc = bf ? launch_attn_fwd_bf16(sh, S, &qr, &kr, v, o, lse, scale, st)
                    : launch_attn_fwd_f32(sh, S, &qr, &kr, v, o, lse, scale, st);
  timer_end(stop, st);
  return rc;
}

// workspace: [q_rot | k_rot] (rope) | lse2_pad | delta_pad | dq_acc (bf16) ;
//            deterministic bf16: dq_acc replaced by the per-K/V-tile dQ
//            partials (n_kv_tiles, B, H, S_pad, D) ;
//            [q_rot | k_rot | dq_rot | dk_rot] (rope) | delta (f32)
size_t fa_bwd_workspace_bytes(int dtype, int B, int S, int H, int D,
                              const fa_rope_t* rope, int deterministic) {
  const size_t n = (size_t)B * S * H * D;
  if (dtype == FA_DTYPE_BF16) {
    const size_t s_pad = (size_t)((S + 127) / 128) * 128;
    size_t total = rope_table_bytes(S, rope);
    if (rope) total += 2 * align256(n * 2);
    total += 2 * align256((size_t)B * H * s_pad * 4);
    const size_t acc = (size_t)B * H * s_pad * D * 4;  // one (B, H, S_pad, D) fp32 array
    total += align256(deterministic ? (s_pad / 128) * acc : acc);
    return total;
  }
  size_t total = rope_table_bytes(S, rope);
  if (rope) total += 4 * align256(n * 4);
  total += align256((size_t)B * H * S * 4);
  return total;
}

int fa_bwd(int dtype, int B, int S, int H, int D, const fa_tensor_t* q,
           const fa_tensor_t* k, const fa_tensor_t* v, const fa_tensor_t* o,
           const fa_tensor_t* d_o, const float* lse, const fa_tensor_t* dq,
           const fa_tensor_t* dk, const fa_tensor_t* dv, float scale,
           const fa_rope_t* rope, int deterministic, void* workspace,
           size_t workspace_bytes, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  FA_TRY(check_rope(rope, D));
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  const bool bf = dtype == FA_DTYPE_BF16;
  const int es = bf ? 2 : 4;
  for (const fa_tensor_t* t : {q, k, v, d_o}) FA_TRY(check_tensor(t, es, bf));
  for (const fa_tensor_t* t : {o, dq, dk, dv}) FA_TRY(check_tensor(t, es, true));
  if (lse == nullptr) return FA_ERR_INVALID_ARG;
  FA_TRY(check_sm100());
  const size_t need = fa_bwd_workspace_bytes(dtype, B, S, H, D, rope, deterministic);
  if (workspace == nullptr || workspace_bytes < need) return FA_ERR_WORKSPACE;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const AttnShape sh{B, S, H, D};
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const size_t n = (size_t)B * S * H * D;
  fa_tensor_t qr = *q, kr = *k;
  float2* table = nullptr;
  if (rope) {
    table = reinterpret_cast<float2*>(ws);
    ws += rope_table_bytes(S, rope);
  }
  if (bf) {
    if (rope) {
      qr = contiguous_view(ws, S, H, D);
      ws += align256(n * 2);
      kr = contiguous_view(ws, S, H, D);
      ws += align256(n * 2);
      // the rotation pass also writes the (cos, sin) table the dK epilogue
      // and the dQ finish read
      FA_TRY(launch_rope_pair(dtype, sh, q, &qr, k, &kr, rope, 0, 0, st, nullptr, table));
    }
    const int s_pad = ((S + 127) / 128) * 128;
    float* lse2 = reinterpret_cast<float*>(ws);
    ws += align256((size_t)B * H * s_pad * 4);
    float* delta = reinterpret_cast<float*>(ws);
    ws += align256((size_t)B * H * s_pad * 4);
    float* dq_acc = reinterpret_cast<float*>(ws);
    if (deterministic) {
      // every K/V tile's dQ contribution lands in its own slot (plain
      // stores, nothing to clear), summed in slot order by the finish pass
      FA_TRY(launch_bwd_delta(dtype, sh, o, d_o, lse, delta, lse2, s_pad, st));
      cudaEvent_t stop = timer_begin(FA_TIMER_BWD, st);
      const int rc = launch_attn_bwd_bf16(sh, S, &qr, &kr, v, d_o, lse2, delta, nullptr, dk, dv,
                                          nullptr, nullptr, 0, scale, rope, table, st, nullptr,
                                          dq_acc);
      timer_end(stop, st);
      FA_TRY(rc);
      return launch_dq_parts_finish(dtype, sh, dq_acc, s_pad / 128,
                                    (int64_t)B * H * s_pad * D, s_pad, dq, scale, rope, table,
                                    st);
    }
    // Delta / LSE2 prologue; it also clears the dQ accumulator
    FA_TRY(launch_bwd_delta(dtype, sh, o, d_o, lse, delta, lse2, s_pad, st, dq_acc));
    cudaEvent_t stop = timer_begin(FA_TIMER_BWD, st);
    const int rc = launch_attn_bwd_bf16(sh, S, &qr, &kr, v, d_o, lse2, delta,
                                        dq_acc, dk, dv, nullptr, nullptr, 0, scale,
                                        rope, table, st);
    timer_end(stop, st);
    FA_TRY(rc);
    return launch_cast_f32(dtype, sh, dq_acc, dq, scale, rope, 0, st, table, s_pad);
  }
  // fp32 path
  fa_tensor_t dqr = *dq, dkr = *dk;
  if (rope) {
    qr = contiguous_view(ws, S, H, D);
    ws += align256(n * 4);
    kr = contiguous_view(ws, S, H, D);
    ws += align256(n * 4);
    dqr = contiguous_view(ws, S, H, D);
    ws += align256(n * 4);
    dkr = contiguous_view(ws, S, H, D);
    ws += align256(n * 4);
    FA_TRY(launch_rope_pair(dtype, sh, q, &qr, k, &kr, rope, 0, 0, st, nullptr, table));
  }
  float* delta = reinterpret_cast<float*>(ws);
  FA_TRY(launch_bwd_delta(dtype, sh, o, d_o, lse, delta, nullptr, S, st));
  cudaEvent_t stop = timer_begin(FA_TIMER_BWD, st);
  const int rc = launch_attn_bwd_f32(sh, &qr, &kr, v, d_o, lse, delta, &dqr,
                                     &dkr, dv, scale, st);
  timer_end(stop, st);
  FA_TRY(rc);
  if (rope) FA_TRY(launch_rope_pair(dtype, sh, &dqr, dq, &dkr, dk, rope, 1, 0, st, table));
  return FA_OK;
}

size_t fa_bwd_saved_workspace_bytes(int dtype, int B, int S, int H, int D) {
  if (dtype != FA_DTYPE_BF16) return 0;
  const size_t s_pad = (size_t)((S + 127) / 128) * 128;
  return 2 * align256((size_t)B * H * s_pad * 4) + align256((size_t)B * H * s_pad * D * 4);
}

int fa_bwd_saved(int dtype, int B, int S, int H, int D, const void* fwd_workspace,
                 size_t fwd_workspace_bytes, const fa_tensor_t* v, const fa_tensor_t* o,
                 const fa_tensor_t* d_o, const float* lse, const fa_tensor_t* dq,
                 const fa_tensor_t* dk, const fa_tensor_t* dv, float scale,
                 const fa_rope_t* rope, void* workspace, size_t workspace_bytes,
                 void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (rope == nullptr) return FA_ERR_INVALID_ARG;  // without RoPE call fa_bwd
  FA_TRY(check_rope(rope, D));
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  FA_TRY(check_tensor(v, 2, true));
  FA_TRY(check_tensor(d_o, 2, true));
  for (const fa_tensor_t* t : {o, dq, dk, dv}) FA_TRY(check_tensor(t, 2, true));
  if (lse == nullptr || fwd_workspace == nullptr) return FA_ERR_INVALID_ARG;
  if (fwd_workspace_bytes < fa_fwd_workspace_bytes(dtype, B, S, H, D, rope))
    return FA_ERR_WORKSPACE;
  if (workspace == nullptr || workspace_bytes < fa_bwd_saved_workspace_bytes(dtype, B, S, H, D))
    return FA_ERR_WORKSPACE;
  FA_TRY(check_sm100());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const AttnShape sh{B, S, H, D};
  // the forward's rotated q, k and (cos, sin) table
  uint8_t* fws = reinterpret_cast<uint8_t*>(const_cast<void*>(fwd_workspace));
  const size_t tb = align256((size_t)B * S * H * D * 2);
  const fa_tensor_t qr = contiguous_view(fws, S, H, D);
  const fa_tensor_t kr = contiguous_view(fws + tb, S, H, D);
  const float2* table = reinterpret_cast<const float2*>(fws + 2 * tb);
  const int s_pad = ((S + 127) / 128) * 128;
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  float* lse2 = reinterpret_cast<float*>(ws);
  ws += align256((size_t)B * H * s_pad * 4);
  float* delta = reinterpret_cast<float*>(ws);
  ws += align256((size_t)B * H * s_pad * 4);
  float* dq_acc = reinterpret_cast<float*>(ws);
  FA_TRY(launch_bwd_delta(dtype, sh, o, d_o, lse, delta, lse2, s_pad, st, dq_acc));
  cudaEvent_t stop = timer_begin(FA_TIMER_BWD, st);
  const int rc = launch_attn_bwd_bf16(sh, S, &qr, &kr, v, d_o, lse2, delta, dq_acc, dk, dv,
                                      nullptr, nullptr, 0, scale, rope, table, st);
  timer_end(stop, st);
  FA_TRY(rc);
  return launch_cast_f32(dtype, sh, dq_acc, dq, scale, rope, 0, st, table, s_pad);
}

// ------------------------------------------------------------ QK prologue
static int check_qk_prologue(int dtype, int B, int T, int I, int H, int D,
                             const fa_tensor_t* x_txt, const fa_tensor_t* x_img,
                             const void* w_txt, const void* w_img, float eps,
                             const fa_rope_t* rope) {
  if (dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (D != 128) return FA_ERR_UNSUPPORTED;
  if (B <= 0 || H <= 0 || H > 24 || T < 0 || I < 0 || T + I <= 0) return FA_ERR_INVALID_ARG;
  if ((int64_t)B * (T + I) * H > (int64_t)1 << 31) return FA_ERR_TOO_LARGE;
  if (!(eps >= 0.f) || !std::isfinite(eps)) return FA_ERR_INVALID_ARG;
  if (rope != nullptr && (rope->axis_dim != 32 || rope->n_axes != 4)) return FA_ERR_UNSUPPORTED;
  FA_TRY(check_rope(rope, D));
  // weights: both streams' (RMSNorm) or none (rotation and concatenation only)
  const bool norm = (T > 0 ? w_txt : w_img) != nullptr;
  if (T > 0) {
    FA_TRY(check_tensor(x_txt, 2, true));
    if ((w_txt != nullptr) != norm) return FA_ERR_INVALID_ARG;
    if (norm && reinterpret_cast<uintptr_t>(w_txt) % 16 != 0) return FA_ERR_ALIGNMENT;
  }
  if (I > 0) {
    FA_TRY(check_tensor(x_img, 2, true));
    if ((w_img != nullptr) != norm) return FA_ERR_INVALID_ARG;
    if (norm && reinterpret_cast<uintptr_t>(w_img) % 16 != 0) return FA_ERR_ALIGNMENT;
  }
  return FA_OK;
}

int fa_qk_norm_rope_fwd(int dtype, int B, int T, int I, int H, int D,
                        const fa_tensor_t* x_txt, const fa_tensor_t* x_img,
                        const void* w_txt, const void* w_img, float eps,
                        const fa_rope_t* rope, const fa_tensor_t* y, void* stream) {
  FA_TRY(check_qk_prologue(dtype, B, T, I, H, D, x_txt, x_img, w_txt, w_img, eps, rope));
  FA_TRY(check_tensor(y, 2, true));
  FA_TRY(check_sm100());
  return launch_qk_norm_rope_fwd(B, T, I, H, x_txt, x_img, w_txt, w_img, eps, rope, y,
                                 reinterpret_cast<cudaStream_t>(stream));
}

int fa_qk_norm_rope_bwd(int dtype, int B, int T, int I, int H, int D,
                        const fa_tensor_t* x_txt, const fa_tensor_t* x_img,
                        const void* w_txt, const void* w_img, float eps,
                        const fa_rope_t* rope, const fa_tensor_t* dy,
                        const fa_tensor_t* dx_txt, const fa_tensor_t* dx_img,
                        float* dw_txt, float* dw_img, void* stream) {
  FA_TRY(check_qk_prologue(dtype, B, T, I, H, D, x_txt, x_img, w_txt, w_img, eps, rope));
  FA_TRY(check_tensor(dy, 2, true));
  if (T > 0) FA_TRY(check_tensor(dx_txt, 2, true));
  if (I > 0) FA_TRY(check_tensor(dx_img, 2, true));
  FA_TRY(check_sm100());
  return launch_qk_norm_rope_bwd(B, T, I, H, x_txt, x_img, w_txt, w_img, eps, rope, dy, dx_txt,
                                 dx_img, dw_txt, dw_img, reinterpret_cast<cudaStream_t>(stream));
}

int fa_rope_apply(int dtype, int B, int S, int H, int D, const fa_tensor_t* x,
                  const fa_tensor_t* y, const fa_rope_t* rope, int inverse,
                  void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (rope == nullptr) return FA_ERR_INVALID_ARG;
  FA_TRY(check_rope(rope, D));
  const int es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  FA_TRY(check_tensor(x, es, false));
  FA_TRY(check_tensor(y, es, false));
  FA_TRY(check_sm100());
  return launch_rope(dtype, AttnShape{B, S, H, D}, x, y, rope, inverse, 0,
                     reinterpret_cast<cudaStream_t>(stream));
}

int fa_fwd_partial(int dtype, int B, int S, int kv_len, int H, int D,
                   const fa_tensor_t* q, const fa_tensor_t* k,
                   const fa_tensor_t* v, const fa_tensor_t* o_blk,
                   float* lse_blk, float scale, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (kv_len <= 0) return FA_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  const bool bf = dtype == FA_DTYPE_BF16;
  const int es = bf ? 2 : 4;
  for (const fa_tensor_t* t : {q, k, v}) FA_TRY(check_tensor(t, es, bf));
  FA_TRY(check_tensor(o_blk, es, true));
  if (lse_blk == nullptr) return FA_ERR_INVALID_ARG;
  FA_TRY(check_sm100());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const AttnShape sh{B, S, H, D};
  cudaEvent_t stop = timer_begin(FA_TIMER_FWD, st);
  const int rc = bf ? launch_attn_fwd_bf16(sh, kv_len, q, k, v, o_blk, lse_blk, scale, st)
                    : launch_attn_fwd_f32(sh, kv_len, q, k, v, o_blk, lse_blk, scale, st);
  timer_end(stop, st);
  return rc;
}

int fa_fwd_fold(int dtype, int B, int S, int kv_len, int H, int D,
                const fa_tensor_t* q, const fa_tensor_t* k, const fa_tensor_t* v,
                float* o_acc, float* lse_acc, int step, int last,
                const fa_tensor_t* o, float* lse, float scale, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;  // fp32: fa_fwd_partial + fa_lse_merge
  if (kv_len <= 0 || step < 0) return FA_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  for (const fa_tensor_t* t : {q, k, v}) FA_TRY(check_tensor(t, 2, true));
  const int mode = step == 0 ? (last ? 0 : 1) : (last ? 3 : 2);
  if (mode != 0 && (o_acc == nullptr || lse_acc == nullptr)) return FA_ERR_INVALID_ARG;
  if (mode != 0 && reinterpret_cast<uintptr_t>(o_acc) % 16 != 0) return FA_ERR_ALIGNMENT;
  if (last) {
    FA_TRY(check_tensor(o, 2, true));
    if (lse == nullptr) return FA_ERR_INVALID_ARG;
  }
  FA_TRY(check_sm100());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaEvent_t stop = timer_begin(FA_TIMER_FWD, st);
  const int rc = launch_attn_fwd_bf16(AttnShape{B, S, H, D}, kv_len, q, k, v, last ? o : nullptr,
                                      lse, scale, st, mode, o_acc, lse_acc);
  timer_end(stop, st);
  return rc;
}

int fa_lse_merge(int dtype, int B, int S, int H, int D, float* o_acc,
                 float* lse_acc, const fa_tensor_t* o_blk,
                 const float* lse_blk, int first, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (!o_acc || !lse_acc || !lse_blk) return FA_ERR_INVALID_ARG;
  FA_TRY(check_tensor(o_blk, dtype == FA_DTYPE_BF16 ? 2 : 4, false));
  FA_TRY(check_sm100());
  return launch_lse_merge(dtype, AttnShape{B, S, H, D}, o_acc, lse_acc, o_blk,
                          lse_blk, first, reinterpret_cast<cudaStream_t>(stream));
}

int fa_bwd_prepare(int dtype, int B, int S, int H, int D, const fa_tensor_t* o,
                   const fa_tensor_t* d_o, const float* lse, float* lse2_pad,
                   float* delta_pad, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  const int es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  FA_TRY(check_tensor(o, es, false));
  FA_TRY(check_tensor(d_o, es, false));
  if (lse == nullptr || lse2_pad == nullptr || delta_pad == nullptr) return FA_ERR_INVALID_ARG;
  FA_TRY(check_sm100());
  const int s_pad = ((S + 127) / 128) * 128;
  return launch_bwd_delta(dtype, AttnShape{B, S, H, D}, o, d_o, lse, delta_pad,
                          lse2_pad, s_pad, reinterpret_cast<cudaStream_t>(stream));
}

int fa_bwd_partial(int dtype, int B, int S, int kv_len, int H, int D,
                   const fa_tensor_t* q, const fa_tensor_t* k,
                   const fa_tensor_t* v, const fa_tensor_t* d_o,
                   const float* lse2_pad, const float* delta_pad, float* dq_acc,
                   float* dk_acc, float* dv_acc, int accumulate, float scale,
                   void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (kv_len <= 0) return FA_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  for (const fa_tensor_t* t : {q, k, v, d_o}) FA_TRY(check_tensor(t, 2, true));
  if (!lse2_pad || !delta_pad || !dq_acc || !dk_acc || !dv_acc) return FA_ERR_INVALID_ARG;
  for (const void* pp : {(const void*)lse2_pad, (const void*)delta_pad, (const void*)dq_acc,
                         (const void*)dk_acc, (const void*)dv_acc})
    if (reinterpret_cast<uintptr_t>(pp) % 16 != 0) return FA_ERR_ALIGNMENT;
  FA_TRY(check_sm100());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaEvent_t stop = timer_begin(FA_TIMER_BWD, st);
  const int rc = launch_attn_bwd_bf16(AttnShape{B, S, H, D}, kv_len, q, k, v, d_o, lse2_pad,
                                      delta_pad, dq_acc, nullptr, nullptr, dk_acc, dv_acc,
                                      accumulate, scale, nullptr, nullptr, st);
  timer_end(stop, st);
  return rc;
}

int fa_add_f32(int64_t n, float* dst, const float* src, void* stream) {
  if (n < 0 || (n > 0 && (dst == nullptr || src == nullptr))) return FA_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(dst) % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0)
    return FA_ERR_ALIGNMENT;
  if (n == 0) return FA_OK;
  FA_TRY(check_sm100());
  return launch_add_f32(n, dst, src, reinterpret_cast<cudaStream_t>(stream));
}

int fa_cast_f32(int dtype, int B, int S, int H, int D, const float* x,
                int x_layout, const fa_tensor_t* y, float alpha,
                const fa_rope_t* rope, void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  FA_TRY(check_rope(rope, D));
  if (x == nullptr || (x_layout != 0 && x_layout != 1)) return FA_ERR_INVALID_ARG;
  FA_TRY(check_tensor(y, dtype == FA_DTYPE_BF16 ? 2 : 4, false));
  FA_TRY(check_sm100());
  const int s_pad = x_layout == 1 ? ((S + 127) / 128) * 128 : 0;
  return launch_cast_f32(dtype, AttnShape{B, S, H, D}, x, y, alpha, rope, 0,
                         reinterpret_cast<cudaStream_t>(stream), nullptr, s_pad);
}

// ------------------------------------------------------------ peer exchange

size_t fa_peer_flags_bytes(void) { return 256; }

int fa_peer_alloc(size_t bytes, void** ptr, fa_peer_handle_t* handle) {
  if (bytes == 0 || ptr == nullptr || handle == nullptr) return FA_ERR_INVALID_ARG;
  FA_TRY(check_sm100());
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return record_cuda_error(e);
  cudaIpcMemHandle_t h;
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return record_cuda_error(e);
  }
  static_assert(sizeof(h) == sizeof(handle->bytes), "IPC handle size");
  std::memcpy(handle->bytes, &h, sizeof(h));
  *ptr = p;
  return FA_OK;
}

int fa_peer_open(const fa_peer_handle_t* handle, void** ptr) {
  if (handle == nullptr || ptr == nullptr) return FA_ERR_INVALID_ARG;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle->bytes, sizeof(h));
  void* p = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return record_cuda_error(e);
  *ptr = p;
  return FA_OK;
}

int fa_peer_close(void* ptr) {
  if (ptr == nullptr) return FA_ERR_INVALID_ARG;
  return record_cuda_error(cudaIpcCloseMemHandle(ptr));
}

int fa_peer_free(void* ptr) {
  if (ptr == nullptr) return FA_ERR_INVALID_ARG;
  return record_cuda_error(cudaFree(ptr));
}

int fa_copy_2d(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
               size_t height, void* stream) {
  if (width == 0 || height == 0) return FA_OK;
  if (dst == nullptr || src == nullptr || dpitch < width || spitch < width)
    return FA_ERR_INVALID_ARG;
  const cudaError_t e = cudaMemcpy2DAsync(dst, dpitch, src, spitch, width, height,
                                          cudaMemcpyDefault,
                                          reinterpret_cast<cudaStream_t>(stream));
  return record_cuda_error(e);
}

int fa_copy_2d_sm(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                  size_t height, int ctas, void* stream) {
  if (width == 0 || height == 0) return FA_OK;
  if (dst == nullptr || src == nullptr || dpitch < width || spitch < width || ctas < 1)
    return FA_ERR_INVALID_ARG;
  if (width % 16 != 0 || dpitch % 16 != 0 || spitch % 16 != 0 ||
      reinterpret_cast<uintptr_t>(dst) % 16 != 0 || reinterpret_cast<uintptr_t>(src) % 16 != 0)
    return FA_ERR_ALIGNMENT;
  if (height > 65535) return FA_ERR_TOO_LARGE;  // one grid row per copied row
  FA_TRY(check_sm100());
  return launch_copy2d_sm(dst, dpitch, src, spitch, width, height, ctas,
                          reinterpret_cast<cudaStream_t>(stream));
}

int fa_peer_barrier(int rank, int world, void* const* flags, int channel, double timeout_s,
                    void* stream) {
  if (world < 1 || world > FA_PEER_MAX || rank < 0 || rank >= world || flags == nullptr ||
      channel < 0 || channel >= FA_PEER_CHANNELS || !(timeout_s > 0.0))
    return FA_ERR_INVALID_ARG;
  for (int i = 0; i < world; ++i)
    if (flags[i] == nullptr || reinterpret_cast<uintptr_t>(flags[i]) % 16 != 0)
      return FA_ERR_INVALID_ARG;
  if (world == 1) return FA_OK;
  FA_TRY(check_sm100());
  return launch_peer_barrier(rank, world, flags, channel, timeout_s,
                             reinterpret_cast<cudaStream_t>(stream));
}

int fa_bwd_scatter(int dtype, int B, int S, int kv_len, int H, int D, const fa_tensor_t* q,
                   const fa_tensor_t* k, const fa_tensor_t* v, const fa_tensor_t* d_o,
                   const float* lse2_pad, const float* delta_pad, float* dq_acc, int seg,
                   int n_seg, float* const* dk_seg, float* const* dv_seg, float scale,
                   void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (dtype != FA_DTYPE_BF16) return FA_ERR_UNSUPPORTED;
  if (kv_len <= 0 || seg <= 0 || n_seg < 1 || n_seg > FA_PEER_MAX ||
      (int64_t)seg * n_seg < kv_len || (int64_t)seg * (n_seg - 1) >= kv_len)
    return FA_ERR_INVALID_ARG;
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  for (const fa_tensor_t* t : {q, k, v, d_o}) FA_TRY(check_tensor(t, 2, true));
  if (!lse2_pad || !delta_pad || !dq_acc || !dk_seg || !dv_seg) return FA_ERR_INVALID_ARG;
  for (const void* pp : {(const void*)lse2_pad, (const void*)delta_pad, (const void*)dq_acc})
    if (reinterpret_cast<uintptr_t>(pp) % 16 != 0) return FA_ERR_ALIGNMENT;
  BwdScatter sc{};
  sc.seg = seg;
  sc.n = n_seg;
  for (int i = 0; i < n_seg; ++i) {
    if (dk_seg[i] == nullptr || dv_seg[i] == nullptr) return FA_ERR_INVALID_ARG;
    if (reinterpret_cast<uintptr_t>(dk_seg[i]) % 16 != 0 ||
        reinterpret_cast<uintptr_t>(dv_seg[i]) % 16 != 0)
      return FA_ERR_ALIGNMENT;
    sc.dk[i] = dk_seg[i];
    sc.dv[i] = dv_seg[i];
  }
  FA_TRY(check_sm100());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  cudaEvent_t stop = timer_begin(FA_TIMER_BWD, st);
  const int rc = launch_attn_bwd_bf16(AttnShape{B, S, H, D}, kv_len, q, k, v, d_o, lse2_pad,
                                      delta_pad, dq_acc, nullptr, nullptr, nullptr, nullptr, 0,
                                      scale, nullptr, nullptr, st, &sc);
  timer_end(stop, st);
  return rc;
}

int fa_reduce_cast_f32(int dtype, int B, int S, int H, int D, const float* x, const float* x2,
                       int n_parts, int64_t part_stride, const fa_tensor_t* y,
                       const fa_tensor_t* y2, float alpha, const fa_rope_t* rope,
                       void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  FA_TRY(check_rope(rope, D));
  if (D != 128) return FA_ERR_UNSUPPORTED;
  if (rope != nullptr && (rope->axis_dim != 32 || rope->n_axes != 4)) return FA_ERR_UNSUPPORTED;
  if (x == nullptr || n_parts < 1 || part_stride < (int64_t)B * S * H * D ||
      part_stride % 4 != 0 || (y2 != nullptr && x2 == nullptr))
    return FA_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(x) % 16 != 0 ||
      (x2 != nullptr && reinterpret_cast<uintptr_t>(x2) % 16 != 0))
    return FA_ERR_ALIGNMENT;
  const int es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  for (const fa_tensor_t* t : {y, y2}) {
    if (t == nullptr) continue;
    FA_TRY(check_tensor(t, es, false));
    if (reinterpret_cast<uintptr_t>(t->data) % 16 != 0 ||
        (t->stride_b * es) % 16 != 0 || (t->stride_s * es) % 16 != 0 ||
        (t->stride_h * es) % 16 != 0)
      return FA_ERR_ALIGNMENT;
  }
  FA_TRY(check_sm100());
  return launch_reduce_cast(dtype, AttnShape{B, S, H, D}, x, x2, n_parts, part_stride, y, y2,
                            alpha, rope, reinterpret_cast<cudaStream_t>(stream));
}

int fa_merge_f32(int dtype, int B, int S, int H, int D, const float* o_a, const float* lse_a,
                 const float* o_b, const float* lse_b, const fa_tensor_t* o, float* lse,
                 void* stream) {
  FA_TRY(check_attn_shape(dtype, B, S, H, D));
  if (D != 128) return FA_ERR_UNSUPPORTED;
  if (!o_a || !lse_a || !o_b || !lse_b || !lse) return FA_ERR_INVALID_ARG;
  if (reinterpret_cast<uintptr_t>(o_a) % 16 != 0 || reinterpret_cast<uintptr_t>(o_b) % 16 != 0)
    return FA_ERR_ALIGNMENT;
  const int es = dtype == FA_DTYPE_BF16 ? 2 : 4;
  FA_TRY(check_tensor(o, es, false));
  if (reinterpret_cast<uintptr_t>(o->data) % 16 != 0 || (o->stride_b * es) % 16 != 0 ||
      (o->stride_s * es) % 16 != 0 || (o->stride_h * es) % 16 != 0)
    return FA_ERR_ALIGNMENT;
  FA_TRY(check_sm100());
  return launch_merge2(dtype, AttnShape{B, S, H, D}, o_a, lse_a, o_b, lse_b, o, lse,
                       reinterpret_cast<cudaStream_t>(stream));
}

int fa_timing_enable(int on) {
  g_timing.store(on ? 1 : 0, std::memory_order_relaxed);
  return FA_OK;
}

int fa_timing_read(int kernel, double* total_ms, int* launches) {
  if (kernel < 0 || kernel >= FA_TIMER_COUNT || !total_ms || !launches)
    return FA_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_timer_mu);
  TimerSlot& s = g_slots[kernel];
  double total = 0.0;
  for (size_t i = 0; i < s.used; ++i) {
    if (cudaEventSynchronize(s.pairs[i].second) != cudaSuccess) return FA_ERR_LAUNCH;
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, s.pairs[i].first, s.pairs[i].second) != cudaSuccess)
      return FA_ERR_LAUNCH;
    total += ms;
  }
  *total_ms = total;
  *launches = (int)s.used;
  s.used = 0;
  return FA_OK;
}

}  // extern "C"
