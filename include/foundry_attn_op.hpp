// foundry_attn_op.hpp — C++ host mirror of the reference's attention custom op.
//
// The reference is Rust on Candle: `struct AttnBwd; impl CustomOp3 for AttnBwd`
// (crates/foundry-spike/src/lib.rs:151-264) with name() / cpu_fwd / cuda_fwd /
// bwd, invoked as `q.apply_op3(&k, &v, AttnBwd)` (lib.rs:366, 444). This header
// keeps that surface in C++ over the C ABI of foundry_attn.h, for hosts that
// are C++ (and as the shape a Rust `impl CustomOp3` over the same C ABI takes):
//   * storages are owned by the caller's allocator, as Candle owns them; the op
//     returns freshly allocated outputs (lib.rs:185, 212);
//   * errors are values (Result), like candle_core::Result / bail!;
//   * layouts are arbitrary strided (B,S,H,D) or (S,H,D) views: no copies are
//     made (the reference materialises contiguous copies, lib.rs:200-207);
//   * cuda_fwd keeps the fp32 log-sum-exp for bwd (the reference recomputes
//     softmax in bwd, lib.rs:232-238); cpu_fwd always fails: the B200 op has no
//     CPU fallback.
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <cmath>
#include <cstdint>
#include <memory>
#include <mutex>
#include <optional>
#include <string>
#include <tuple>
#include <utility>

#include "foundry_attn.h"

namespace foundry {

enum class DType { F32, BF16 };

inline int dtype_code(DType d) { return d == DType::BF16 ? FA_DTYPE_BF16 : FA_DTYPE_F32; }
inline size_t dtype_size(DType d) { return d == DType::BF16 ? 2 : 4; }

// Result<T>: a value or an error message (candle_core::Result analogue).
template <typename T>
struct Result {
  std::optional<T> value;
  std::string error;
  static Result ok(T v) { return Result{std::move(v), {}}; }
  static Result err(std::string e) { return Result{std::nullopt, std::move(e)}; }
  bool is_ok() const { return value.has_value(); }
};

// Device allocation interface (the framework owns storage, as Candle does).
struct Allocator {
  virtual ~Allocator() = default;
  virtual void* allocate(size_t bytes) = 0;
  virtual void release(void* p) = 0;
};

// Default: cudaMalloc / cudaFree on the current device.
struct CudaAllocator final : Allocator {
  void* allocate(size_t bytes) override {
    void* p = nullptr;
    return cudaMalloc(&p, bytes) == cudaSuccess ? p : nullptr;
  }
  void release(void* p) override { cudaFree(p); }
};

// A device buffer released through its allocator.
struct CudaStorage {
  std::shared_ptr<void> ptr;
  size_t bytes = 0;
  DType dtype = DType::BF16;
  void* data() const { return ptr.get(); }
  static std::optional<CudaStorage> make(Allocator& a, size_t bytes, DType d) {
    void* p = a.allocate(bytes);
    if (p == nullptr) return std::nullopt;
    CudaStorage s;
    s.ptr = std::shared_ptr<void>(p, [&a](void* q) { a.release(q); });
    s.bytes = bytes;
    s.dtype = d;
    return s;
  }
};

// Shape and element strides of a (B,S,H,D) view; (S,H,D) has B = 1.
struct Layout {
  std::array<int64_t, 4> shape{1, 1, 1, 1};
  std::array<int64_t, 4> stride{0, 0, 0, 1};
  int64_t offset = 0;  // in elements
  static Layout contiguous(int64_t B, int64_t S, int64_t H, int64_t D) {
    Layout l;
    l.shape = {B, S, H, D};
    l.stride = {S * H * D, H * D, D, 1};
    return l;
  }
  int64_t numel() const { return shape[0] * shape[1] * shape[2] * shape[3]; }
};

struct DeviceTensor {
  CudaStorage storage;
  Layout layout;
  void* ptr() const {
    return static_cast<uint8_t*>(storage.data()) + layout.offset * dtype_size(storage.dtype);
  }
  fa_tensor_t desc() const {
    return fa_tensor_t{ptr(), layout.stride[0], layout.stride[1], layout.stride[2],
                       layout.stride[3]};
  }
};

// The op. Mirrors `AttnBwd` (lib.rs:151-264).
class AttnBwd {
 public:
  struct Rope {
    const float* pos = nullptr;  // device (S, n_axes) fp32
    int n_axes = 4;
    int axis_dim = 32;
    float theta = 10000.f;
  };

  explicit AttnBwd(Allocator& alloc, std::optional<float> scale = std::nullopt,
                   std::optional<Rope> rope = std::nullopt, cudaStream_t stream = nullptr)
      : alloc_(alloc), scale_(scale), rope_(rope), stream_(stream) {}

  const char* name() const { return "foundry-attn-bwd"; }  // lib.rs:154-156

  // lib.rs:158-187 runs the reference arithmetic on the CPU; the B200 op does not.
  Result<DeviceTensor> cpu_fwd(const DeviceTensor&, const DeviceTensor&,
                               const DeviceTensor&) const {
    return Result<DeviceTensor>::err(
        "foundry-attn-bwd: no CPU path; the op runs on sm_100 devices only");
  }

  // lib.rs:189-214. Returns a fresh output; keeps the LSE for bwd.
  Result<DeviceTensor> cuda_fwd(const DeviceTensor& q, const DeviceTensor& k,
                                const DeviceTensor& v) {
    if (auto e = check_same(q, k, v)) return Result<DeviceTensor>::err(*e);
    const auto& s = q.layout.shape;
    const DType dt = q.storage.dtype;
    auto out_st = CudaStorage::make(alloc_, q.layout.numel() * dtype_size(dt), dt);
    auto lse_st = CudaStorage::make(alloc_, s[0] * s[2] * s[1] * sizeof(float), DType::F32);
    if (!out_st || !lse_st) return Result<DeviceTensor>::err("foundry-attn-bwd: out of memory");
    DeviceTensor out{*out_st, Layout::contiguous(s[0], s[1], s[2], s[3])};
    fa_rope_t r = rope_struct();
    const fa_rope_t* rp = rope_ ? &r : nullptr;
    const size_t ws_bytes = fa_fwd_workspace_bytes(dtype_code(dt), (int)s[0], (int)s[1],
                                                   (int)s[2], (int)s[3], rp);
    std::optional<CudaStorage> ws;
    if (ws_bytes) {
      ws = CudaStorage::make(alloc_, ws_bytes, DType::F32);
      if (!ws) return Result<DeviceTensor>::err("foundry-attn-bwd: out of memory");
    }
    fa_tensor_t dq = q.desc(), dk = k.desc(), dv = v.desc(), dout = out.desc();
    const int rc = fa_fwd(dtype_code(dt), (int)s[0], (int)s[1], (int)s[2], (int)s[3], &dq, &dk,
                          &dv, &dout, static_cast<float*>(lse_st->data()), scale(s[3]), rp,
                          ws ? ws->data() : nullptr, ws_bytes, stream_);
    if (rc != FA_OK) return Result<DeviceTensor>::err(std::string("fa_fwd: ") + fa_status_string(rc));
    std::lock_guard<std::mutex> lk(mu_);
    saved_lse_ = lse_st;
    return Result<DeviceTensor>::ok(out);
  }

  // lib.rs:216-263: (dq, dk, dv) from q, k, v, the forward output and its gradient.
  using Grads = std::tuple<DeviceTensor, DeviceTensor, DeviceTensor>;
  Result<Grads> bwd(const DeviceTensor& q, const DeviceTensor& k, const DeviceTensor& v,
                    const DeviceTensor& res, const DeviceTensor& grad_res) {
    if (auto e = check_same(q, k, v)) return Result<Grads>::err(*e);
    std::optional<CudaStorage> lse;
    {
      std::lock_guard<std::mutex> lk(mu_);
      lse = saved_lse_;
    }
    if (!lse) {
      auto again = cuda_fwd(q, k, v);  // rebuild the statistics
      if (!again.is_ok()) return Result<Grads>::err(again.error);
      std::lock_guard<std::mutex> lk(mu_);
      lse = saved_lse_;
    }
    const auto& s = q.layout.shape;
    const DType dt = q.storage.dtype;
    const size_t bytes = q.layout.numel() * dtype_size(dt);
    auto a = CudaStorage::make(alloc_, bytes, dt);
    auto b = CudaStorage::make(alloc_, bytes, dt);
    auto c = CudaStorage::make(alloc_, bytes, dt);
    if (!a || !b || !c) return Result<Grads>::err("foundry-attn-bwd: out of memory");
    const Layout lc = Layout::contiguous(s[0], s[1], s[2], s[3]);
    DeviceTensor gq{*a, lc}, gk{*b, lc}, gv{*c, lc};
    fa_rope_t r = rope_struct();
    const fa_rope_t* rp = rope_ ? &r : nullptr;
    const size_t ws_bytes = fa_bwd_workspace_bytes(dtype_code(dt), (int)s[0], (int)s[1],
                                                   (int)s[2], (int)s[3], rp, 0);
    auto ws = CudaStorage::make(alloc_, ws_bytes ? ws_bytes : 16, DType::F32);
    if (!ws) return Result<Grads>::err("foundry-attn-bwd: out of memory");
    fa_tensor_t tq = q.desc(), tk = k.desc(), tv = v.desc(), to = res.desc(),
                tdo = grad_res.desc(), tdq = gq.desc(), tdk = gk.desc(), tdv = gv.desc();
    const int rc = fa_bwd(dtype_code(dt), (int)s[0], (int)s[1], (int)s[2], (int)s[3], &tq, &tk,
                          &tv, &to, &tdo, static_cast<const float*>(lse->data()), &tdq, &tdk,
                          &tdv, scale(s[3]), rp, 0, ws->data(), ws_bytes, stream_);
    if (rc != FA_OK) return Result<Grads>::err(std::string("fa_bwd: ") + fa_status_string(rc));
    // keep the workspace alive until the stream has consumed it
    if (cudaStreamSynchronize(stream_) != cudaSuccess)
      return Result<Grads>::err("fa_bwd: stream synchronisation failed");
    return Result<Grads>::ok(Grads{gq, gk, gv});
  }

 private:
  std::optional<std::string> check_same(const DeviceTensor& q, const DeviceTensor& k,
                                        const DeviceTensor& v) const {
    if (q.layout.shape != k.layout.shape || q.layout.shape != v.layout.shape)
      return std::string("foundry-attn-bwd: q, k, v shapes differ");
    if (q.storage.dtype != k.storage.dtype || q.storage.dtype != v.storage.dtype)
      return std::string("foundry-attn-bwd: q, k, v dtypes differ");
    return std::nullopt;
  }
  float scale(int64_t d) const { return scale_ ? *scale_ : (float)(1.0 / std::sqrt((double)d)); }
  fa_rope_t rope_struct() const {
    fa_rope_t r{};
    if (rope_) r = fa_rope_t{rope_->pos, rope_->n_axes, rope_->axis_dim, rope_->theta};
    return r;
  }

  Allocator& alloc_;
  std::optional<float> scale_;
  std::optional<Rope> rope_;
  cudaStream_t stream_;
  std::mutex mu_;
  std::optional<CudaStorage> saved_lse_;
};

}  // namespace foundry
