// attn_common.h — host-side helpers shared by the attention launchers:
// shapes, TMA descriptor encoding for strided (B, S, H, D) tensors, and the
// per-device shared-memory attribute cache.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "foundry_attn.h"

namespace fa {

struct AttnShape {
  int B, S, H, D;
};

// Encodes a 4-D TMA descriptor over a bf16 (B, S, H, D) tensor with box
// (64 head-dim elements, box_rows tokens, 1, 1), SWIZZLE_128B, zero fill out
// of bounds. Returns FA_OK or an FA_ERR_* code.
int make_tmap_bshd(CUtensorMap* map, const fa_tensor_t* t, int B, int S, int H,
                   int D, int box_rows);

// Same over an fp32 (B, S, H, D) tensor with box (32, box_rows, 1, 1).
int make_tmap_bshd_f32(CUtensorMap* map, const fa_tensor_t* t, int B, int S,
                       int H, int D, int box_rows);

enum KernelId {
  kKernelFwdBf16 = 0,
  kKernelBwdBf16 = 1,
  kKernelF32Fwd = 2,
  kKernelF32Bwd = 3,
  kKernelCount = 8
};

// FA_OK when the last CUDA runtime call / launch on this thread succeeded;
// otherwise records the CUDA error text (see fa_last_error) and returns
// FA_ERR_LAUNCH.
int launch_status();
int record_cuda_error(cudaError_t e);
// Sets the text fa_last_error() returns on this thread.
void record_error_text(const char* msg);

// Shape rules every attention entry point shares: dtype F32 or BF16, positive
// sizes, head_dim 128, B and H within a grid dimension, B*S*H*D < 2^40.
int check_attn_shape(int dtype, int B, int S, int H, int D);

// Raises the dynamic shared-memory limit of `fn` once per (device, kernel).
int ensure_smem_attr(const void* fn, int bytes, int kernel_id);

// bf16 sm_100a kernels
// merge: 0 plain; 1 (o_acc, lse_acc) <- block; 2 fold block into them;
// 3 fold, then write o (bf16) and lse (see the kernel's Params)
// In-tile rotation of q and k (axial RoPE, four 32-wide axes): the kernel
// rotates each Q and K tile in shared memory as it lands and writes the
// rotated q and k to q_rot / k_rot ((B, S, H, D) bf16) for the backward.
// Each K tile is rotated once: the CTA that owns it publishes it to k_rot
// and sets its flag; other CTAs load the published copy when its flag is
// set and otherwise rotate the raw tile themselves (nobody waits).
struct FwdRope {
  const uint32_t* cs;  // packed bf16 (cos, sin), (S, 64) words
  const fa_tensor_t* q_rot;
  const fa_tensor_t* k_rot;
  uint32_t* k_pub;     // (B, H, ceil(S/128)) flags, zero before the launch
};

int launch_attn_fwd_bf16(const AttnShape& sh, int kv_len, const fa_tensor_t* q,
                         const fa_tensor_t* k, const fa_tensor_t* v,
                         const fa_tensor_t* o, float* lse, float scale,
                         cudaStream_t stream, int merge = 0, float* o_acc = nullptr,
                         float* lse_acc = nullptr, const FwdRope* rope = nullptr);

// dK/dV rows stored per key segment: row j to dk[j / seg], dv[j / seg] at
// local row j % seg (fp32 contiguous (B, seg, H, D) each; peers' memory allowed)
struct BwdScatter {
  int seg, n;
  float* dk[FA_PEER_MAX];
  float* dv[FA_PEER_MAX];
};

int launch_attn_bwd_bf16(const AttnShape& sh, int kv_len, const fa_tensor_t* q,
                         const fa_tensor_t* k, const fa_tensor_t* v,
                         const fa_tensor_t* d_o, const float* lse2_pad,
                         const float* delta_pad, float* dq_acc,
                         const fa_tensor_t* dk, const fa_tensor_t* dv,
                         float* dk_acc, float* dv_acc, int accumulate, float scale,
                         const fa_rope_t* rope, const float2* rope_table,
                         cudaStream_t stream, const BwdScatter* scatter = nullptr,
                         float* dq_part = nullptr);

// fp32 SIMT kernels (exact path)
int launch_attn_fwd_f32(const AttnShape& sh, int kv_len, const fa_tensor_t* q,
                        const fa_tensor_t* k, const fa_tensor_t* v,
                        const fa_tensor_t* o, float* lse, float scale,
                        cudaStream_t stream);
int launch_attn_bwd_f32(const AttnShape& sh, const fa_tensor_t* q,
                        const fa_tensor_t* k, const fa_tensor_t* v,
                        const fa_tensor_t* d_o, const float* lse,
                        const float* delta, const fa_tensor_t* dq,
                        const fa_tensor_t* dk, const fa_tensor_t* dv,
                        float scale, cudaStream_t stream);

// elementwise helpers (misc.cu)
// delta[b,h,s] = sum_d dO*O over rows s < s_pad (0 for s >= S); when lse2 is
// non-null also lse2[b,h,s] = lse*log2(e) (+inf for s >= S).
// zero_acc: an fp32 (B, H, s_pad, D) buffer cleared on the way (or nullptr)
int launch_bwd_delta(int dtype, const AttnShape& sh, const fa_tensor_t* o,
                     const fa_tensor_t* d_o, const float* lse, float* delta,
                     float* lse2, int s_pad, cudaStream_t stream,
                     float* zero_acc = nullptr);
// (cos, sin) table for tokens [0, S) (+pos_offset), S * n_axes*axis_dim/2 float2
int launch_rope_table(int dtype, int S, const fa_rope_t* rope, int pos_offset,
                      float2* table, cudaStream_t stream);
// bf16 path: the float2 table and the packed bf16 (cos, sin) words (cos in
// bits 0-15, sin in bits 16-31), S * n_axes*axis_dim/2 entries each
// (it also zeroes `n_clear` words at `clear`: the forward's publish flags)
int launch_rope_table2(int S, const fa_rope_t* rope, float2* table, uint32_t* packed,
                       uint32_t* clear, int64_t n_clear, cudaStream_t stream);
// table may be nullptr (cos/sin evaluated per element)
int launch_rope(int dtype, const AttnShape& sh, const fa_tensor_t* x,
                const fa_tensor_t* y, const fa_rope_t* rope, int inverse,
                int pos_offset, cudaStream_t stream, const float2* table = nullptr);
// table: (cos, sin) to read, or nullptr to evaluate them; table_out: where
// the token-major path also writes the evaluated values (nullptr: nowhere)
int launch_rope_pair(int dtype, const AttnShape& sh, const fa_tensor_t* x0,
                     const fa_tensor_t* y0, const fa_tensor_t* x1,
                     const fa_tensor_t* y1, const fa_rope_t* rope, int inverse,
                     int pos_offset, cudaStream_t stream, const float2* table,
                     float2* table_out = nullptr);
// x: fp32 (B, S, H, D) contiguous, or (B, H, s_pad, D) when s_pad > 0
int launch_cast_f32(int dtype, const AttnShape& sh, const float* x,
                    const fa_tensor_t* y, float alpha, const fa_rope_t* rope,
                    int pos_offset, cudaStream_t stream, const float2* table = nullptr,
                    int s_pad = 0);
// dQ of the deterministic bf16 backward: y = alpha * inverse_rope(sum over
// j < n_parts of x[j]) in index order; x fp32 (n_parts, B, H, s_pad, D),
// parts part_stride floats apart (rope may be nullptr; table as above)
int launch_dq_parts_finish(int dtype, const AttnShape& sh, const float* x, int n_parts,
                           int64_t part_stride, int s_pad, const fa_tensor_t* y, float alpha,
                           const fa_rope_t* rope, const float2* table, cudaStream_t stream);
// dst[i] += src[i], i < n
int launch_add_f32(int64_t n, float* dst, const float* src, cudaStream_t stream);
int launch_lse_merge(int dtype, const AttnShape& sh, float* o_acc,
                     float* lse_acc, const fa_tensor_t* o_blk,
                     const float* lse_blk, int first, cudaStream_t stream);

// QK prologue (qk_prologue.cu): per stream RMSNorm + RoPE into the joint
// (B, T+I, H, 128) tensor, and its backward (dw_* accumulated, may be null)
int launch_qk_norm_rope_fwd(int B, int T, int I, int H, const fa_tensor_t* x_txt,
                            const fa_tensor_t* x_img, const void* w_txt, const void* w_img,
                            float eps, const fa_rope_t* rope, const fa_tensor_t* y,
                            cudaStream_t stream);
int launch_qk_norm_rope_bwd(int B, int T, int I, int H, const fa_tensor_t* x_txt,
                            const fa_tensor_t* x_img, const void* w_txt, const void* w_img,
                            float eps, const fa_rope_t* rope, const fa_tensor_t* dy,
                            const fa_tensor_t* dx_txt, const fa_tensor_t* dx_img, float* dw_txt,
                            float* dw_img, cudaStream_t stream);

// Sequence-parallel exchange (peer.cu): bounded barrier over the ranks' flag
// blocks, the owner's sum of received dK/dV contributions (dK un-rotated and
// scaled by alpha), and the merge of two fp32 (O, LSE) partials
int launch_peer_barrier(int rank, int world, void* const* flags, int channel,
                        double timeout_s, cudaStream_t stream);
int launch_copy2d_sm(void* dst, size_t dpitch, const void* src, size_t spitch, size_t width,
                     size_t height, int ctas, cudaStream_t stream);
int launch_reduce_cast(int dtype, const AttnShape& sh, const float* x, const float* x2,
                       int n_parts, int64_t part_stride, const fa_tensor_t* y,
                       const fa_tensor_t* y2, float alpha, const fa_rope_t* rope,
                       cudaStream_t stream);
int launch_merge2(int dtype, const AttnShape& sh, const float* o_a, const float* lse_a,
                  const float* o_b, const float* lse_b, const fa_tensor_t* o, float* lse,
                  cudaStream_t stream);

// Host: read-and-clear the device status word of each kernel translation
// unit (0: no bounded wait expired; -1: unreadable).
int fwd_device_status();
int bwd_device_status();
int f32_device_status();
int misc_device_status();
int qkp_device_status();
int peer_device_status();

}  // namespace fa
