// test_attn_op.cpp — drives the C++ CustomOp3 mirror (foundry_attn_op.hpp) the
// way the reference drives its op (src/bin/attn_backward.rs:203-233): forward,
// then bwd seeded with an upstream gradient. Inputs and outputs are raw fp32
// files so the Python test can check them against the CPU oracle.
//
//   test_attn_op <dir> <f32|bf16> <S> <H> [rope]
// reads <dir>/{q,k,v,do}.bin (S*H*128 fp32, (S,H,D) order) and, with "rope",
// <dir>/pos.bin (S*4 fp32); writes <dir>/{o,dq,dk,dv}.bin (fp32).
#include <cuda_bf16.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "foundry_attn_op.hpp"

using foundry::AttnBwd;
using foundry::CudaAllocator;
using foundry::CudaStorage;
using foundry::DeviceTensor;
using foundry::DType;
using foundry::Layout;

static std::vector<float> read_f32(const std::string& path, size_t n) {
  std::vector<float> v(n);
  FILE* f = std::fopen(path.c_str(), "rb");
  if (!f || std::fread(v.data(), 4, n, f) != n) {
    std::fprintf(stderr, "cannot read %s\n", path.c_str());
    std::exit(2);
  }
  std::fclose(f);
  return v;
}

static void write_f32(const std::string& path, const std::vector<float>& v) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f || std::fwrite(v.data(), 4, v.size(), f) != v.size()) {
    std::fprintf(stderr, "cannot write %s\n", path.c_str());
    std::exit(2);
  }
  std::fclose(f);
}

static DeviceTensor upload(CudaAllocator& a, const std::vector<float>& h, DType dt, int S,
                           int H) {
  const size_t n = h.size();
  auto st = CudaStorage::make(a, n * foundry::dtype_size(dt), dt);
  if (!st) std::exit(3);
  if (dt == DType::F32) {
    cudaMemcpy(st->data(), h.data(), n * 4, cudaMemcpyHostToDevice);
  } else {
    std::vector<__nv_bfloat16> b(n);
    for (size_t i = 0; i < n; ++i) b[i] = __float2bfloat16_rn(h[i]);
    cudaMemcpy(st->data(), b.data(), n * 2, cudaMemcpyHostToDevice);
  }
  return DeviceTensor{*st, Layout::contiguous(1, S, H, 128)};
}

static std::vector<float> download(const DeviceTensor& t) {
  const size_t n = t.layout.numel();
  std::vector<float> out(n);
  if (t.storage.dtype == DType::F32) {
    cudaMemcpy(out.data(), t.ptr(), n * 4, cudaMemcpyDeviceToHost);
  } else {
    std::vector<__nv_bfloat16> b(n);
    cudaMemcpy(b.data(), t.ptr(), n * 2, cudaMemcpyDeviceToHost);
    for (size_t i = 0; i < n; ++i) out[i] = __bfloat162float(b[i]);
  }
  return out;
}

int main(int argc, char** argv) {
  if (argc < 5) {
    std::fprintf(stderr, "usage: %s <dir> <f32|bf16> <S> <H> [rope]\n", argv[0]);
    return 2;
  }
  const std::string dir = argv[1];
  const DType dt = std::string(argv[2]) == "bf16" ? DType::BF16 : DType::F32;
  const int S = std::atoi(argv[3]), H = std::atoi(argv[4]);
  const bool with_rope = argc > 5 && std::string(argv[5]) == "rope";
  const size_t n = (size_t)S * H * 128;
  CudaAllocator alloc;
  DeviceTensor q = upload(alloc, read_f32(dir + "/q.bin", n), dt, S, H);
  DeviceTensor k = upload(alloc, read_f32(dir + "/k.bin", n), dt, S, H);
  DeviceTensor v = upload(alloc, read_f32(dir + "/v.bin", n), dt, S, H);
  DeviceTensor d_o = upload(alloc, read_f32(dir + "/do.bin", n), dt, S, H);
  std::optional<AttnBwd::Rope> rope;
  std::optional<CudaStorage> pos_st;
  if (with_rope) {
    auto pos = read_f32(dir + "/pos.bin", (size_t)S * 4);
    pos_st = CudaStorage::make(alloc, pos.size() * 4, DType::F32);
    cudaMemcpy(pos_st->data(), pos.data(), pos.size() * 4, cudaMemcpyHostToDevice);
    AttnBwd::Rope r;
    r.pos = static_cast<const float*>(pos_st->data());
    rope = r;
  }
  AttnBwd op(alloc, std::nullopt, rope);
  if (std::string(op.name()) != "foundry-attn-bwd") return 4;
  if (op.cpu_fwd(q, k, v).is_ok()) return 5;  // no CPU fallback
  auto out = op.cuda_fwd(q, k, v);
  if (!out.is_ok()) {
    std::fprintf(stderr, "%s\n", out.error.c_str());
    return 6;
  }
  auto grads = op.bwd(q, k, v, *out.value, d_o);
  if (!grads.is_ok()) {
    std::fprintf(stderr, "%s\n", grads.error.c_str());
    return 7;
  }
  if (cudaDeviceSynchronize() != cudaSuccess || fa_device_status() != 0) return 8;
  write_f32(dir + "/o.bin", download(*out.value));
  write_f32(dir + "/dq.bin", download(std::get<0>(*grads.value)));
  write_f32(dir + "/dk.bin", download(std::get<1>(*grads.value)));
  write_f32(dir + "/dv.bin", download(std::get<2>(*grads.value)));
  std::printf("ok\n");
  return 0;
}
