// noalloc.cu — the bf16 backward with its scratch in a static device array.
//
// fa_bwd needs a caller-provided workspace (the fp32 dQ accumulator and two
// per-row tables). Some callers cannot hand one over: a framework whose
// memory pool already owns the device memory and offers no raw allocation
// at this call site, or a code path where cudaMalloc's implicit device-wide
// synchronisation is not acceptable. fa_bwd_noalloc runs the same kernels
// with that scratch taken from a file-scope __device__ array of
// kNoAllocScratchBytes instead; it calls no allocator at all.
//
// Costs and rules of the static array:
//   * every GPU that loads this library holds kNoAllocScratchBytes of device
//     memory from module load until process exit;
//   * all calls on a device share the one array and it keeps the previous
//     call's contents (the dQ accumulator is cleared at the start of every
//     call); calls whose work overlaps on the GPU (different streams without
//     ordering between them) race on the array and give wrong results;
//   * host code cannot use the array's name as a device address: the address
//     comes from cudaGetSymbolAddress, taken by the first call on a device
//     (with that device current), which should therefore come before any
//     stream capture. The address is cached per device together with the
//     CUDA context it was taken in; after a cudaDeviceReset the next call
//     sees a new context and looks the address up again.
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "attn_common.h"

namespace fa {

constexpr size_t kNoAllocScratchBytes = size_t(64) << 20;  // 64 MiB per device

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

static std::mutex g_noalloc_mu;
static void* g_noalloc_ptr[64];      // device address of the array, per device
static CUcontext g_noalloc_ctx[64];  // the context that address belongs to

// The calling thread's current driver context (nullptr when the driver entry
// point is unavailable; the cached address is then never invalidated).
static CUcontext current_context() {
  static PFN_cuCtxGetCurrent_v4000 get = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(fn);
  });
  CUcontext ctx = nullptr;
  if (get != nullptr && get(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  return ctx;
}

// Device address of the static scratch on the current device (looked up on
// the first call for that device, and again when its context was re-created).
static int noalloc_scratch(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return FA_ERR_NO_DEVICE;
  const CUcontext ctx = current_context();  // nullptr before the runtime made one
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr || g_noalloc_ctx[dev] != ctx) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return record_cuda_error(e);
    g_noalloc_ptr[dev] = p;
    g_noalloc_ctx[dev] = current_context();  // the lookup made the context current
  }
  *out = g_noalloc_ptr[dev];
  return FA_OK;
}

static size_t round256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace fa

using namespace fa;

extern "C" int fa_bwd_noalloc(int B, int S, int H, int D, const fa_tensor_t* q,
                              const fa_tensor_t* k, const fa_tensor_t* v,
                              const fa_tensor_t* o, const fa_tensor_t* d_o,
                              const float* lse, const fa_tensor_t* dq,
                              const fa_tensor_t* dk, const fa_tensor_t* dv,
                              float scale, void* stream) {
  int rc = check_attn_shape(FA_DTYPE_BF16, B, S, H, D);
  if (rc != FA_OK) return rc;
  if (!(scale > 0.f) || !std::isfinite(scale)) return FA_ERR_INVALID_ARG;
  for (const fa_tensor_t* t : {q, k, v, o, d_o, dq, dk, dv}) {
    if (t == nullptr || t->data == nullptr) return FA_ERR_INVALID_ARG;
    if (t->stride_d != 1 || reinterpret_cast<uintptr_t>(t->data) % 16 != 0)
      return FA_ERR_ALIGNMENT;
  }
  if (lse == nullptr) return FA_ERR_INVALID_ARG;
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
      major != 10)
    return FA_ERR_NO_DEVICE;
  // scratch: LSE*log2(e) and Delta padded to 128-row tiles, fp32 dQ accumulator
  const int64_t s_pad64 = ((int64_t)S + 127) / 128 * 128;
  const size_t rows = (size_t)B * (size_t)H * (size_t)s_pad64;
  const size_t need = 2 * round256(rows * 4) + round256(rows * D * 4);
  if (need > kNoAllocScratchBytes) {
    record_error_text("fa_bwd_noalloc: B*H*ceil(S/128)*128 rows need more scratch than the "
                      "64 MiB static array holds; use fa_bwd with a caller workspace");
    return FA_ERR_TOO_LARGE;
  }
  const int s_pad = (int)s_pad64;  // fits: the rows fit the 64 MiB array
  void* base = nullptr;
  rc = noalloc_scratch(&base);
  if (rc != FA_OK) return rc;
  uint8_t* ws = static_cast<uint8_t*>(base);
  float* lse2 = reinterpret_cast<float*>(ws);
  float* delta = reinterpret_cast<float*>(ws + round256(rows * 4));
  float* dq_acc = reinterpret_cast<float*>(ws + 2 * round256(rows * 4));
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const AttnShape sh{B, S, H, D};
  // the array keeps the previous call's sums: the Delta pass clears the
  // accumulator on its way
  rc = launch_bwd_delta(FA_DTYPE_BF16, sh, o, d_o, lse, delta, lse2, s_pad, st, dq_acc);
  if (rc != FA_OK) return rc;
  rc = launch_attn_bwd_bf16(sh, S, q, k, v, d_o, lse2, delta, dq_acc, dk, dv,
                            nullptr, nullptr, 0, scale, nullptr, nullptr, st);
  if (rc != FA_OK) return rc;
  return launch_cast_f32(FA_DTYPE_BF16, sh, dq_acc, dq, scale, nullptr, 0, st,
                         nullptr, s_pad);
}
