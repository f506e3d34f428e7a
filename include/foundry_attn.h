/*
 * foundry_attn.h — C ABI of the B200 (sm_100a) joint text+image attention op.
 *
 * This is the drop-in boundary for foundry-trainer's attention custom op
 * `AttnBwd` (crates/foundry-spike/src/lib.rs:151-264). A host binding (a Rust
 * FFI crate over these declarations, the C++ mirror in foundry_attn_op.hpp,
 * or the Python ctypes mirror) calls these entry points; nothing here uses
 * torch or any other framework type.
 *
 * Conventions (all entry points):
 *   - Tensors are (B, S, H, D) with arbitrary element strides (fa_tensor_t);
 *     the reference's op is the B == 1 case with (S, H, D) inputs (lib.rs:134).
 *     The head-dim stride must be 1; other strides times the element size must
 *     be multiples of 16 bytes and base pointers 16-byte aligned (TMA rules).
 *   - The caller owns every buffer, including workspaces; nothing allocates.
 *   - Calls are asynchronous and ordered on `stream` (a cudaStream_t; NULL is
 *     the legacy default stream).
 *   - Errors are status codes (FA_OK == 0); nothing throws across the ABI.
 *     fa_status_string() names a code. Device-side bounded waits that expire
 *     report FA_ERR_DEVICE_TIMEOUT through fa_device_status().
 *   - Reentrant. The only global state is a per-device, call-once cache of the
 *     driver entry point used to encode TMA descriptors, and the device status
 *     word.
 */
#ifndef FOUNDRY_ATTN_H
#define FOUNDRY_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FA_ABI_VERSION 1

/* status codes */
#define FA_OK 0
#define FA_ERR_INVALID_ARG 1     /* null pointer, non-positive size, bad scale */
#define FA_ERR_UNSUPPORTED 2     /* dtype / head_dim / rope layout not supported */
#define FA_ERR_ALIGNMENT 3       /* stride or base pointer violates the TMA rules */
#define FA_ERR_LAUNCH 4          /* a CUDA launch or runtime call failed */
#define FA_ERR_DEVICE_TIMEOUT 5  /* a device-side bounded wait expired */
#define FA_ERR_WORKSPACE 6       /* workspace missing or too small */
#define FA_ERR_NO_DEVICE 7       /* no sm_100 device current */
#define FA_ERR_TOO_LARGE 8       /* size beyond the kernel's addressing limits */

/* element types; the reference's compute dtypes are f32 and bf16 (lib.rs:139-147) */
#define FA_DTYPE_F32 0
#define FA_DTYPE_BF16 1

/* A strided (B, S, H, D) device tensor. Strides are in elements. */
typedef struct {
  void* data;
  int64_t stride_b;
  int64_t stride_s;
  int64_t stride_h;
  int64_t stride_d;
} fa_tensor_t;

/*
 * Axial rotary embedding, the reference's rope_tables_dtype + apply_rope
 * (lib.rs:77-129): per token a position vector of n_axes floats; axis a owns
 * head-dim segment [a*axis_dim, (a+1)*axis_dim); frequency j < axis_dim/2 is
 * theta^(-2j/axis_dim); rotate-half inside each segment. cos/sin are computed
 * in fp32 and rounded to the compute dtype before use, as the reference does.
 * `pos` is a device pointer to a (S, n_axes) fp32 array shared by the batch.
 * Supported: n_axes * axis_dim == D, axis_dim even.
 */
typedef struct {
  const float* pos;
  int n_axes;
  int axis_dim;
  float theta;
} fa_rope_t;

/*
 * Forward. Replaces AttnBwd::cuda_fwd (lib.rs:189-214) / attn_fwd
 * (lib.rs:133-149): O = softmax(Q K^T * scale) V, non-causal, no mask.
 * Also writes the per-row log-sum-exp `lse` (fp32, contiguous (B, H, S),
 * natural log of sum exp(scaled scores)) that fa_bwd consumes; the reference
 * recomputes it instead (lib.rs:232-238).
 * If `rope` is non-NULL, q and k are pre-rotation and the rotation is applied
 * inside the op (the reference applies it before the op, lib.rs:326-358).
 * `workspace` (may be NULL when fa_fwd_workspace_bytes() returns 0) receives
 * the rotated q and k and their (cos, sin) table, which fa_bwd_saved can
 * reuse.
 */
int fa_fwd(int dtype, int B, int S, int H, int D,
           const fa_tensor_t* q, const fa_tensor_t* k, const fa_tensor_t* v,
           const fa_tensor_t* o, float* lse, float scale, const fa_rope_t* rope,
           void* workspace, size_t workspace_bytes, void* stream);

size_t fa_fwd_workspace_bytes(int dtype, int B, int S, int H, int D,
                              const fa_rope_t* rope);

/*
 * Backward. Replaces AttnBwd::bwd (lib.rs:216-263): given q, k, v, the
 * forward output o, its gradient d_o and the saved lse, writes dq, dk, dv
 * (w.r.t. the pre-rotation q/k when `rope` is non-NULL).
 * `deterministic` != 0 requests bit-identical results across repeats
 * (the reference's stability gate, bin/stability.rs:177-189: identical bits
 * across repeat runs, docs/TESTING.md:19); the f32 path is always
 * deterministic. The bf16 path then stores each 128-key tile's dQ
 * contribution in its own fp32 slot and sums the slots in a fixed order
 * instead of adding them into one accumulator in arrival order: its
 * workspace grows to B*H*ceil(S/128)*S_pad*D*4 bytes (S_pad = S rounded up
 * to 128; 2 GB at B1 H24 S4608) and the sum is one extra pass over it.
 * `workspace` must hold fa_bwd_workspace_bytes(); it carries the fp32 dQ
 * accumulator (or the partials) and the per-row softmax-gradient term.
 */
int fa_bwd(int dtype, int B, int S, int H, int D,
           const fa_tensor_t* q, const fa_tensor_t* k, const fa_tensor_t* v,
           const fa_tensor_t* o, const fa_tensor_t* d_o, const float* lse,
           const fa_tensor_t* dq, const fa_tensor_t* dk, const fa_tensor_t* dv,
           float scale, const fa_rope_t* rope, int deterministic,
           void* workspace, size_t workspace_bytes, void* stream);

size_t fa_bwd_workspace_bytes(int dtype, int B, int S, int H, int D,
                              const fa_rope_t* rope, int deterministic);

/*
 * Backward that reuses the forward's rotation (bf16, RoPE inside the op).
 * fa_fwd with `rope` leaves in its workspace the rotated q, k and the
 * (cos, sin) table; passing that workspace here (`fwd_workspace`, untouched
 * since the forward) skips the second rotation of q and k that fa_bwd does.
 * The reference's backward likewise works on the rotated q, k saved as the
 * op's inputs (lib.rs:216-263). Results equal fa_bwd's for the same inputs.
 * `workspace` must hold fa_bwd_saved_workspace_bytes().
 */
int fa_bwd_saved(int dtype, int B, int S, int H, int D,
                 const void* fwd_workspace, size_t fwd_workspace_bytes,
                 const fa_tensor_t* v, const fa_tensor_t* o, const fa_tensor_t* d_o,
                 const float* lse, const fa_tensor_t* dq, const fa_tensor_t* dk,
                 const fa_tensor_t* dv, float scale, const fa_rope_t* rope,
                 void* workspace, size_t workspace_bytes, void* stream);

size_t fa_bwd_saved_workspace_bytes(int dtype, int B, int S, int H, int D);

/*
 * Standalone rotation, the reference's apply_rope (lib.rs:122-129) for
 * callers that rotate outside the op: y = x*cos + rotate_half(x)*sin per axis
 * segment, fp32 arithmetic, result in `dtype`. `inverse` != 0 applies the
 * transposed rotation (the gradient of apply_rope). x and y may alias.
 */
int fa_rope_apply(int dtype, int B, int S, int H, int D, const fa_tensor_t* x,
                  const fa_tensor_t* y, const fa_rope_t* rope, int inverse,
                  void* stream);

/*
 * Q/K prologue of the joint block, fused (bf16, head dim 128): for each
 * stream — text rows [0, T) from x_txt (B, T, H, 128), image rows [T, T+I)
 * from x_img (B, I, H, 128), any strides with a contiguous head dim — the
 * reference's rms_norm with that stream's weight (lib.rs:45-58; w_* are
 * (128,) bf16, eps as NORM_EPS lib.rs:26), then apply_rope with the joint
 * positions (lib.rs:122-129, rope may be NULL), written into the joint
 * y (B, T+I, H, 128): the cat([txt, img]) of lib.rs:363-365 costs nothing.
 * Either stream may be empty (T = 0 is the single-stream block). With both
 * weights NULL there is no normalisation: the rows are only rotated (rope
 * non-NULL) and concatenated — the joint v, or dO from the two streams'
 * output gradients.
 * The backward maps dy (gradient of y) to dx_txt, dx_img and ADDS the norm
 * weights' gradients into dw_txt, dw_img (fp32 (128,), NULL to skip).
 */
int fa_qk_norm_rope_fwd(int dtype, int B, int T, int I, int H, int D,
                        const fa_tensor_t* x_txt, const fa_tensor_t* x_img,
                        const void* w_txt, const void* w_img, float eps,
                        const fa_rope_t* rope, const fa_tensor_t* y, void* stream);
int fa_qk_norm_rope_bwd(int dtype, int B, int T, int I, int H, int D,
                        const fa_tensor_t* x_txt, const fa_tensor_t* x_img,
                        const void* w_txt, const void* w_img, float eps,
                        const fa_rope_t* rope, const fa_tensor_t* dy,
                        const fa_tensor_t* dx_txt, const fa_tensor_t* dx_img,
                        float* dw_txt, float* dw_img, void* stream);

/*
 * Sequence-parallel (ring) building blocks. They have no counterpart in the
 * reference, which is single-GPU (it has no collectives); they let a host
 * driver rotate K/V shards between ranks and fold each block into the local
 * result. q/k passed here are already rotated (fa_rope_apply with the
 * shard's positions).
 *
 * fa_fwd_partial: attention of the S local query rows against one block of
 *   kv_len keys: o_blk = softmax(q k_blk^T * scale) v_blk, normalised over the
 *   block, and its log-sum-exp lse_blk (fp32, contiguous (B,H,S)).
 * fa_lse_merge: (o_acc, lse_acc) <- merge((o_acc, lse_acc), (o_blk, lse_blk));
 *   o_acc fp32 contiguous (B,S,H,D), lse_acc (B,H,S); first != 0 initialises
 *   the accumulator from the block.
 * fa_bwd_prepare: per local row, lse2_pad = lse * log2(e) and
 *   delta_pad = rowsum(dO * O), both fp32 (B, H, S_pad) with
 *   S_pad = ceil(S/128)*128 (padding +inf and 0), from the merged forward
 *   output o, its gradient d_o and the merged lse.
 * fa_bwd_partial: one K/V block of the bf16 backward against the S local rows:
 *   adds dS K (unscaled) into dq_acc (fp32 (B, H, S_pad, D), zeroed by the
 *   caller before the first block) and writes scale*dS^T Q, P^T dO to dk_acc,
 *   dv_acc (fp32 contiguous (B, kv_len, H, D)): added to their contents when
 *   accumulate != 0, stored over them otherwise.
 * fa_add_f32: dst[i] += src[i] for i < n (fp32, both 16-byte aligned); folds
 *   a block's dK/dV into the accumulator that arrived from the previous rank.
 * fa_cast_f32: y = alpha * x converted to `dtype`, un-rotated when rope is
 *   non-NULL; x is fp32 contiguous (B,S,H,D) (x_layout 0) or (B,H,S_pad,D)
 *   (x_layout 1, the dq_acc layout).
 */
int fa_fwd_partial(int dtype, int B, int S, int kv_len, int H, int D,
                   const fa_tensor_t* q, const fa_tensor_t* k,
                   const fa_tensor_t* v, const fa_tensor_t* o_blk,
                   float* lse_blk, float scale, void* stream);
/*
 * fa_fwd_fold (bf16): fa_fwd_partial and fa_lse_merge in one launch. Folds
 * the block's attention into the running fp32 (o_acc (B,S,H,D), lse_acc
 * (B,H,S)) in the kernel's epilogue: step 0 initialises them, later steps
 * fold into them, and with `last` != 0 the folded result is written as the
 * final o (bf16) and lse instead (step 0 with `last`: a single block, o_acc
 * and lse_acc unused).
 */
int fa_fwd_fold(int dtype, int B, int S, int kv_len, int H, int D,
                const fa_tensor_t* q, const fa_tensor_t* k, const fa_tensor_t* v,
                float* o_acc, float* lse_acc, int step, int last,
                const fa_tensor_t* o, float* lse, float scale, void* stream);
int fa_lse_merge(int dtype, int B, int S, int H, int D, float* o_acc,
                 float* lse_acc, const fa_tensor_t* o_blk,
                 const float* lse_blk, int first, void* stream);
int fa_bwd_prepare(int dtype, int B, int S, int H, int D, const fa_tensor_t* o,
                   const fa_tensor_t* d_o, const float* lse, float* lse2_pad,
                   float* delta_pad, void* stream);
int fa_bwd_partial(int dtype, int B, int S, int kv_len, int H, int D,
                   const fa_tensor_t* q, const fa_tensor_t* k,
                   const fa_tensor_t* v, const fa_tensor_t* d_o,
                   const float* lse2_pad, const float* delta_pad, float* dq_acc,
                   float* dk_acc, float* dv_acc, int accumulate, float scale,
                   void* stream);
int fa_add_f32(int64_t n, float* dst, const float* src, void* stream);
int fa_cast_f32(int dtype, int B, int S, int H, int D, const float* x,
                int x_layout, const fa_tensor_t* y, float alpha,
                const fa_rope_t* rope, void* stream);

/*
 * Peer exchange for sequence parallelism inside one node (one process per
 * GPU, W <= FA_PEER_MAX ranks). These replace the ring's send/recv with the
 * GPUs' peer memory; the reference has no multi-GPU path (its op runs on one
 * device, crates/foundry-spike/src/lib.rs:189-263), so they have no
 * counterpart there and exist for the sharded long-sequence configuration.
 *
 * fa_peer_alloc: a zeroed device allocation of `bytes` on the current device
 *   and its 64-byte CUDA IPC handle (to be sent to the other ranks).
 * fa_peer_open: maps another rank's allocation from its handle; fa_peer_close
 *   unmaps it, fa_peer_free releases an allocation of this rank.
 * fa_copy_2d: stream-ordered copy of `height` rows of `width` bytes (pitches
 *   dpitch/spitch) between any two device addresses, peer-mapped ones
 *   included (the copy engines move the data; no SMs are used).
 * fa_copy_2d_sm: the same copy done by `ctas` small CTAs of SMs (16-byte
 *   loads and stores; width, pitches and addresses 16-byte aligned). Each CTA
 *   fits beside one attention CTA on an SM, so it runs under the kernels.
 * fa_peer_barrier: every rank tells every other rank that it reached the
 *   next epoch of `channel` (< FA_PEER_CHANNELS) and waits until all have.
 *   `flags` holds W pointers to the ranks' flag blocks of
 *   fa_peer_flags_bytes() bytes each (zeroed at start; this rank's own block
 *   local, the others peer-mapped). Writes this device issued before the
 *   barrier on `stream` are visible to the peers once it completes. The wait
 *   is bounded by timeout_s; expiry sets FA_ERR_DEVICE_TIMEOUT in
 *   fa_device_status. All ranks must call it the same number of times per
 *   channel.
 * fa_bwd_scatter: fa_bwd_partial over kv_len keys whose dK/dV rows are stored
 *   (fp32, not accumulated) into n_seg separate buffers: key row j goes to
 *   dk_seg[j / seg], dv_seg[j / seg] at local row j % seg, each buffer fp32
 *   contiguous (B, seg, H, D). The buffers may be other GPUs' memory (the
 *   owners of the key rows); the kernel's epilogue stores into them directly.
 * fa_reduce_cast_f32: y = alpha * inverse_rope(sum_p x[p]) and
 *   y2 = sum_p x2[p] (y2 may be NULL), p < n_parts, parts part_stride floats
 *   apart, x and x2 fp32 contiguous (B,S,H,D): the owner's sum of the dK/dV
 *   contributions it received.
 * fa_merge_f32: (o, lse) <- the merge of two partial results over disjoint
 *   key sets, each fp32 normalised o (B,S,H,D) with natural-log lse (B,H,S).
 */
#define FA_PEER_MAX 8
#define FA_PEER_CHANNELS 4
typedef struct {
  unsigned char bytes[64];
} fa_peer_handle_t;
size_t fa_peer_flags_bytes(void);
int fa_peer_alloc(size_t bytes, void** ptr, fa_peer_handle_t* handle);
int fa_peer_open(const fa_peer_handle_t* handle, void** ptr);
int fa_peer_close(void* ptr);
int fa_peer_free(void* ptr);
int fa_copy_2d(void* dst, size_t dpitch, const void* src, size_t spitch,
               size_t width, size_t height, void* stream);
int fa_copy_2d_sm(void* dst, size_t dpitch, const void* src, size_t spitch,
                  size_t width, size_t height, int ctas, void* stream);
int fa_peer_barrier(int rank, int world, void* const* flags, int channel,
                    double timeout_s, void* stream);
int fa_bwd_scatter(int dtype, int B, int S, int kv_len, int H, int D,
                   const fa_tensor_t* q, const fa_tensor_t* k,
                   const fa_tensor_t* v, const fa_tensor_t* d_o,
                   const float* lse2_pad, const float* delta_pad, float* dq_acc,
                   int seg, int n_seg, float* const* dk_seg, float* const* dv_seg,
                   float scale, void* stream);
int fa_reduce_cast_f32(int dtype, int B, int S, int H, int D, const float* x,
                       const float* x2, int n_parts, int64_t part_stride,
                       const fa_tensor_t* y, const fa_tensor_t* y2, float alpha,
                       const fa_rope_t* rope, void* stream);
int fa_merge_f32(int dtype, int B, int S, int H, int D, const float* o_a,
                 const float* lse_a, const float* o_b, const float* lse_b,
                 const fa_tensor_t* o, float* lse, void* stream);

/*
 * Backward without a caller workspace. This entry point has no counterpart in
 * the reference. It is for callers that cannot allocate device memory where
 * they call the op: a host framework whose memory pool already owns the GPU
 * and offers no raw allocation here, or a path on which cudaMalloc's implicit
 * device-wide synchronisation is not acceptable. It computes what fa_bwd
 * computes for dtype FA_DTYPE_BF16 without RoPE and non-deterministic dQ
 * summation, taking its scratch (the fp32 dQ accumulator and two per-row
 * tables) from a 64 MiB array built into the library instead of a workspace;
 * it allocates nothing. Limits and rules:
 *   - B * H * ceil(S/128) * 128 rows must fit the 64 MiB array (about 129k
 *     rows, e.g. B=1, H=24, S <= 5376); larger sizes return FA_ERR_TOO_LARGE
 *     and fa_last_error() says why.
 *   - The array exists once per GPU that loads the library and stays resident
 *     until the process exits.
 *   - The first call on a device looks up the array's device address (with
 *     that device current); make that first call before any stream capture.
 *     After a cudaDeviceReset the device's context is a new one and the next
 *     call looks the address up again (so that call, too, belongs outside a
 *     capture).
 *   - All calls on one device share the array: calls whose GPU work overlaps
 *     (streams without ordering between them) race and corrupt each other's
 *     dQ. The accumulator is cleared at the start of every call.
 */
int fa_bwd_noalloc(int B, int S, int H, int D, const fa_tensor_t* q,
                   const fa_tensor_t* k, const fa_tensor_t* v,
                   const fa_tensor_t* o, const fa_tensor_t* d_o,
                   const float* lse, const fa_tensor_t* dq,
                   const fa_tensor_t* dk, const fa_tensor_t* dv, float scale,
                   void* stream);

/*
 * Measurement hooks (no counterpart in the reference, which only wall-clocks
 * whole steps, bin/throughput.rs:868-873). While enabled, every launch of the
 * main forward (FA_TIMER_FWD) and backward (FA_TIMER_BWD) kernel is bracketed
 * by CUDA events on its stream. fa_timing_read synchronises on the recorded
 * events, returns the summed device time and launch count since the last
 * read, and resets them. Intended for one device per process.
 */
#define FA_TIMER_FWD 0
#define FA_TIMER_BWD 1
#define FA_TIMER_COUNT 2
int fa_timing_enable(int on);
int fa_timing_read(int kernel, double* total_ms, int* launches);

/* Human-readable name of a status code. Never NULL. */
const char* fa_status_string(int status);

/* The CUDA error behind the last FA_ERR_LAUNCH on the calling thread ("" if
 * none). Never NULL. */
const char* fa_last_error(void);

/*
 * Reads and clears the device status word of the current device that the
 * kernels set when a bounded wait expires (0 when clean). Synchronises the
 * current device.
 */
int fa_device_status(void);

/* ABI version (FA_ABI_VERSION) and a build string. */
int fa_abi_version(void);
const char* fa_build_info(void);

#ifdef __cplusplus
}
#endif

#endif /* FOUNDRY_ATTN_H */
