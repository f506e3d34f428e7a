// umma_selftest.cu — known-answer checks of the sm_100a building blocks the
// attention kernels rely on, one 128x128x128 bf16 product per launch:
//   test 0: D = A B^T, A and B K-major in shared memory (the QK^T form)
//   test 1: D = A B,   B MN-major (the PV / P^T dO form)
//   test 2: D = A B,   A in TMEM (written with tcgen05.st), B MN-major
//   test 3: D = A^T B, A MN-major (stored K x M), B MN-major (the dS K form)
//   test 4: D[:, 64:128] = A B[:, 64:128] with N = 64, B MN-major, D at a
//           TMEM column offset of 64
// A and B are row-major 128x128 bf16 in global memory; D is 128x128 fp32.
// Built into its own library (libfa_selftest.so), used only by the tests.
#include <cudaTypedefs.h>

#include "sm100_ptx.cuh"

namespace {

using namespace fa;

constexpr int kTile = 32768;
constexpr int kBlk = 16384;
constexpr int kSmem = 2 * kTile + 1024 + 256;

__global__ void __launch_bounds__(128, 1)
selftest_kernel(const __grid_constant__ CUtensorMap ta,
                const __grid_constant__ CUtensorMap tb,
                const __nv_bfloat16* a_glob, float* d, int test, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + kTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 2 * kTile);
  uint32_t* slot = reinterpret_cast<uint32_t*>(smem + 2 * kTile + 64);
  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(&bars[0], 2 * kTile);
    tma_load_4d(sa, &ta, &bars[0], 0, 0, 0, 0);
    tma_load_4d(sa + kBlk, &ta, &bars[0], 64, 0, 0, 0);
    tma_load_4d(sb, &tb, &bars[0], 0, 0, 0, 0);
    tma_load_4d(sb + kBlk, &tb, &bars[0], 64, 0, 0, 0);
  }
  bool ok = __all_sync(0xffffffffu, mbar_wait(&bars[0], 0));
  const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
  if (test == 2 && ok) {
    // row r of A -> TMEM lane r, columns [128, 192), two bf16 per column
    const int r = threadIdx.x;
    const uint32_t* src = reinterpret_cast<const uint32_t*>(a_glob + r * 128);
    uint32_t v[32];
    for (int half = 0; half < 2; ++half) {
      for (int i = 0; i < 32; ++i) v[i] = src[half * 32 + i];
      tmem_st32(tmem + lane_off + 128 + half * 32, v);
    }
    tmem_wait_st();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && ok) {
    const uint32_t a = smem_u32(sa), b = smem_u32(sb);
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t acc = kk > 0;
      switch (test) {
        case 0:
          umma_ss(tmem, kmajor_desc(a, kk, kBlk), kmajor_desc(b, kk, kBlk),
                  idesc_bf16(128, 128, false, false), acc);
          break;
        case 1:
          umma_ss(tmem, kmajor_desc(a, kk, kBlk), mnmajor_desc(b, kk, kBlk),
                  idesc_bf16(128, 128, false, true), acc);
          break;
        case 2:
          umma_ts(tmem, tmem + 128 + kk * 8, mnmajor_desc(b, kk, kBlk),
                  idesc_bf16(128, 128, false, true), acc);
          break;
        case 3:
          umma_ss(tmem, mnmajor_desc(a, kk, kBlk), mnmajor_desc(b, kk, kBlk),
                  idesc_bf16(128, 128, true, true), acc);
          break;
        case 4:
          umma_ss(tmem + 64, kmajor_desc(a, kk, kBlk),
                  mnmajor_desc(b + kBlk, kk, kBlk),
                  idesc_bf16(128, 64, false, true), acc);
          break;
      }
    }
    umma_commit(&bars[1]);
  }
  if (ok) ok = __all_sync(0xffffffffu, mbar_wait(&bars[1], 0));
  tc_fence_after();
  if (ok) {
    const int r = threadIdx.x;
    for (int cb = 0; cb < 4; ++cb) {
      uint32_t v[32];
      tmem_ld32(tmem + lane_off + cb * 32, v);
      tmem_wait_ld();
      for (int i = 0; i < 32; ++i) d[r * 128 + cb * 32 + i] = __uint_as_float(v[i]);
    }
  } else if (threadIdx.x == 0) {
    *status = 5;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

int make_map(CUtensorMap* m, const void* p) {
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault,
                              &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess)
    return 4;
  auto enc = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  cuuint64_t dims[4] = {128, 128, 1, 1};
  cuuint64_t strides[3] = {256, 256 * 128, 256 * 128};
  cuuint32_t box[4] = {64, 128, 1, 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(p),
                   dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : 3;
}

}  // namespace

extern "C" int fa_selftest_umma(int test, const void* a, const void* b,
                                float* d, int* status, void* stream) {
  if (test < 0 || test > 4 || !a || !b || !d || !status) return 1;
  CUtensorMap ta, tb;
  int rc = make_map(&ta, a);
  if (!rc) rc = make_map(&tb, b);
  if (rc) return rc;
  if (cudaFuncSetAttribute(selftest_kernel,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           kSmem) != cudaSuccess)
    return 4;
  selftest_kernel<<<1, 128, kSmem, reinterpret_cast<cudaStream_t>(stream)>>>(
      ta, tb, reinterpret_cast<const __nv_bfloat16*>(a), d, test, status);
  return cudaGetLastError() == cudaSuccess ? 0 : 4;
}
