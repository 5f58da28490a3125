// Context, memory, op-level and tensor-parallel entry points of the C ABI.
#include "runtime.hpp"

#include <dlfcn.h>
#include <string.h>

#include <algorithm>
#include <vector>

#include "common.cuh"
#include "attention_tc.cuh"
#include "gemm.cuh"
#include "kernels.cuh"

namespace dcpp {

Nccl& Nccl::get() {
  static Nccl n;
  if (n.loaded) return n;
  void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
  if (!h) fail(DCPP_ERR_NCCL, std::string("cannot load NCCL: ") + dlerror());
  auto sym = [&](const char* name) {
    void* p = dlsym(h, name);
    if (!p) fail(DCPP_ERR_NCCL, std::string("NCCL symbol missing: ") + name);
    return p;
  };
  n.GetUniqueId = reinterpret_cast<int (*)(UniqueId*)>(sym("ncclGetUniqueId"));
  n.CommInitRank = reinterpret_cast<int (*)(Comm*, int, UniqueId, int)>(sym("ncclCommInitRank"));
  n.CommDestroy = reinterpret_cast<int (*)(Comm)>(sym("ncclCommDestroy"));
  n.CommAbort = reinterpret_cast<int (*)(Comm)>(sym("ncclCommAbort"));
  n.AllReduce =
      reinterpret_cast<int (*)(const void*, void*, size_t, int, int, Comm, cudaStream_t)>(sym("ncclAllReduce"));
  n.AllGather = reinterpret_cast<int (*)(const void*, void*, size_t, int, Comm, cudaStream_t)>(sym("ncclAllGather"));
  n.GetErrorString = reinterpret_cast<const char* (*)(int)>(sym("ncclGetErrorString"));
  n.loaded = true;
  return n;
}

void Ctx::maybe_inject(const char* entry) {
  if (fault_countdown <= 0 || fault_name != entry) return;
  if (--fault_countdown == 0) {
    fault_name.clear();
    fail(DCPP_ERR_INJECTED, std::string("injected fault in ") + entry);
  }
}

void* Ctx::ensure_scratch(size_t bytes) {
  if (bytes <= scratch_bytes) return scratch;
  if (scratch) cuda_check(cudaFree(scratch), "cudaFree(scratch)");
  scratch = nullptr;
  scratch_bytes = 0;
  if (cudaMalloc(&scratch, bytes) != cudaSuccess) {
    cudaGetLastError();
    fail(DCPP_ERR_OOM, "scratch allocation of " + std::to_string(bytes) + " bytes failed");
  }
  scratch_bytes = bytes;
  return scratch;
}

void* Ctx::ensure_split_ws(size_t bytes) {
  if (bytes <= split_ws_bytes) return split_ws;
  if (split_ws) cuda_check(cudaFree(split_ws), "cudaFree(split workspace)");
  split_ws = nullptr;
  split_ws_bytes = 0;
  if (cudaMalloc(&split_ws, bytes) != cudaSuccess) {
    cudaGetLastError();
    fail(DCPP_ERR_OOM, "split workspace allocation of " + std::to_string(bytes) + " bytes failed");
  }
  split_ws_bytes = bytes;
  return split_ws;
}

void PeerBuffer::open(Ctx& ctx, size_t nbytes) {
  if (local) fail(DCPP_ERR_STATE, "peer buffer already open");
  if (!ctx.comm || ctx.nranks < 2 || ctx.nranks > 8) fail(DCPP_ERR_STATE, "peer buffer needs a TP group of 2..8");
  auto& n = Nccl::get();
  bytes = nbytes;
  if (cudaMalloc(&local, bytes) != cudaSuccess) {
    cudaGetLastError();
    local = nullptr;
    fail(DCPP_ERR_OOM, "peer buffer allocation failed");
  }
  cuda_check(cudaMemsetAsync(local, 0, bytes, ctx.stream), "clear peer buffer");
  cudaIpcMemHandle_t mine;
  cuda_check(cudaIpcGetMemHandle(&mine, local), "cudaIpcGetMemHandle");
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  uint8_t* dev = nullptr;
  cuda_check(cudaMalloc(&dev, hb * (ctx.nranks + 1)), "handle exchange buffer");
  std::vector<uint8_t> all(hb * ctx.nranks);
  try {
    cuda_check(cudaMemcpyAsync(dev + hb * ctx.nranks, &mine, hb, cudaMemcpyHostToDevice, ctx.stream), "copy handle");
    int r = n.AllGather(dev + hb * ctx.nranks, dev, hb, /*ncclUint8*/ 1, ctx.comm, ctx.stream);
    if (r != 0) fail(DCPP_ERR_NCCL, std::string("ncclAllGather: ") + n.GetErrorString(r));
    cuda_check(cudaMemcpyAsync(all.data(), dev, hb * ctx.nranks, cudaMemcpyDeviceToHost, ctx.stream), "copy handles");
    cuda_check(cudaStreamSynchronize(ctx.stream), "handle exchange");
  } catch (...) {
    cudaFree(dev);
    throw;
  }
  cudaFree(dev);
  for (int j = 0; j < ctx.nranks; ++j) {
    if (j == ctx.rank) {
      peer[j] = local;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, all.data() + hb * j, hb);
    void* p = nullptr;
    cuda_check(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    peer[j] = static_cast<uint8_t*>(p);
  }
}

void PeerBuffer::close(Ctx& ctx) {
  if (!local) return;
  cudaStreamSynchronize(ctx.stream);
  for (int j = 0; j < 8; ++j) {
    if (peer[j] && peer[j] != local) cudaIpcCloseMemHandle(peer[j]);
    peer[j] = nullptr;
  }
  // Every rank has unmapped this rank's buffer before it is freed.
  if (ctx.comm) {
    auto& n = Nccl::get();
    float* one = nullptr;
    if (cudaMalloc(&one, sizeof(float)) == cudaSuccess) {
      n.AllReduce(one, one, 1, /*ncclFloat32*/ 7, /*ncclSum*/ 0, ctx.comm, ctx.stream);
      cudaStreamSynchronize(ctx.stream);
      cudaFree(one);
    }
  }
  cudaFree(local);
  local = nullptr;
  bytes = 0;
}

const char* device_error_name(int code) {
  switch (code) {
    case kDevTimeoutFull: return "GEMM consumer timed out waiting for a shared-memory stage";
    case kDevTimeoutEmpty: return "GEMM producer timed out waiting for a free stage";
    case kDevTimeoutAccum: return "GEMM epilogue timed out waiting for an accumulator";
    case kDevTimeoutAccumFree: return "GEMM MMA warp timed out waiting for a drained accumulator";
    case kDevTimeoutDequant: return "GEMM dequant stage handshake timed out";
    case kDevBadShape: return "kernel launched with an unsupported shape";
    case kDevTimeoutAttn: return "attention pipeline wait timed out";
    case kDevTimeoutPeer: return "tensor-parallel barrier timed out waiting for a peer GPU";
    case kDevBadIndex: return "token id outside the embedding table";
    default: return "unknown device error";
  }
}

void Ctx::check_device_error() {
  int h = 0;
  cuda_check(cudaMemcpyAsync(&h, d_err, sizeof(int), cudaMemcpyDeviceToHost, stream), "read error word");
  cuda_check(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
  if (h != 0) {
    cuda_check(cudaMemsetAsync(d_err, 0, sizeof(int), stream), "clear error word");
    fail(h == kDevBadShape ? DCPP_ERR_UNSUPPORTED : (h == kDevBadIndex ? DCPP_ERR_INVALID_ARG : DCPP_ERR_TIMEOUT),
         std::string("device error ") + std::to_string(h) + ": " + device_error_name(h));
  }
}

size_t row_bytes_of(int type, int64_t n) {
  switch (type) {
    case kTypeF32: return static_cast<size_t>(n) * 4;
    case kTypeF16:
    case kTypeBF16: return static_cast<size_t>(n) * 2;
    case kTypeQ8_0:
      if (n % 32) fail(DCPP_ERR_INVALID_ARG, "Q8_0 row length must be a multiple of 32");
      return static_cast<size_t>(n / 32) * 34;
    case kTypeQ4_K:
      if (n % 256) fail(DCPP_ERR_INVALID_ARG, "Q4_K row length must be a multiple of 256");
      return static_cast<size_t>(n / 256) * 144;
    default: fail(DCPP_ERR_UNSUPPORTED, "unsupported ggml type " + std::to_string(type));
  }
}

// y[M,N] = x[M,K] . W^T through the tensor-core GEMM (weights expanded to
// bf16 into the context scratch first).
void gemm_op(Ctx& c, int wtype, const void* w, int64_t N, int64_t K, const uint16_t* x, int64_t M, float* y) {
  if (N <= 0 || K <= 0 || M <= 0) fail(DCPP_ERR_INVALID_ARG, "dcpp_gemm: sizes must be positive");
  if (K % 8) fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm: K must be a multiple of 8");
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2) fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm: size too large");
  (void)row_bytes_of(wtype, K);
  const uint16_t* wb = nullptr;
  if (wtype == kTypeBF16) {
    wb = static_cast<const uint16_t*>(w);
  } else {
    uint16_t* s = static_cast<uint16_t*>(c.ensure_scratch(static_cast<size_t>(N) * K * 2));
    cuda_check(launch_dequant_bf16(wtype, w, N * K, s, c.stream), "dequant weight");
    wb = s;
  }
  CUtensorMap ta, tb;
  cuda_check(make_tmap_bf16(&ta, x, K, M, K, kGemmBM), "tensor map (x)");
  const bool pair = c.use_pair(M);
  cuda_check(make_tmap_bf16(&tb, wb, K, N, K, pair ? 128 : kGemmBN), "tensor map (W)");
  GemmArgs a{};
  a.N = static_cast<int32_t>(N);
  a.K = static_cast<int32_t>(K);
  a.n_groups = 1;
  a.groups[0].row0 = 0;
  a.groups[0].orow0 = 0;
  a.groups[0].rows = static_cast<int32_t>(M);
  a.ep.mode = kEpiF32;
  a.ep.out_f32 = y;
  a.ep.ld_out = N;
  a.err = c.d_err;
  gemm_finalize_groups(a, pair ? 256 : kGemmBM);
  // Few tiles for the 74 CTA pairs (small M): K slices into f32 partials,
  // then an ordered reduce into y.  Only for a large modelled gain: measured
  // on the config-5 sweep, modest ones (M 1024, K 9216) did not materialise.
  int splits = 1;
  if (pair && N % 4 == 0)
    splits = gemm_choose_k_splits(a.total_tiles, c.num_sms, M, N, K, 8, 8, /*reduce_adds=*/false, 0.4);
  if (splits > 1) {
    a.ep.out_f32 = static_cast<float*>(c.ensure_split_ws(static_cast<size_t>(splits) * M * N * 4));
    gemm_set_k_splits(a, splits, M * N);
  }
  if (pair)
    cuda_check(launch_gemm_pair(ta, tb, tb, a, kBSrcBf16, c.num_sms, c.stream), "launch gemm (pair)");
  else
    cuda_check(launch_gemm(ta, tb, tb, a, kBSrcBf16, c.num_sms, c.stream), "launch gemm");
  if (splits > 1)
    cuda_check(launch_split_reduce(a.ep.out_f32, splits, M * N, M, N, N, y, N, c.stream, /*add=*/false),
               "split reduce");
}

}  // namespace dcpp

using dcpp::Ctx;
using dcpp::Error;

namespace {

template <class F>
dcpp_status guarded(dcpp_ctx* ctx, const char* entry, F&& f) {
  if (!ctx) return DCPP_ERR_INVALID_ARG;
  try {
    ctx->maybe_inject(entry);
    int prev = 0;
    if (cudaGetDevice(&prev) == cudaSuccess && prev != ctx->device) cudaSetDevice(ctx->device);
    f();
    return DCPP_OK;
  } catch (const Error& e) {
    ctx->last_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    ctx->last_error = e.what();
    return DCPP_ERR_INVALID_ARG;
  }
}

}  // namespace

extern "C" {

const char* dcpp_version(void) { return "dcpp-b200 0.1 (sm_100a)"; }

dcpp_status dcpp_init(int device, dcpp_ctx** out_ctx) {
  if (!out_ctx) return DCPP_ERR_INVALID_ARG;
  *out_ctx = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) {
    cudaGetLastError();
    return DCPP_ERR_CUDA;
  }
  auto* c = new dcpp_ctx();
  c->device = device;
  if (cudaSetDevice(device) != cudaSuccess) { delete c; return DCPP_ERR_CUDA; }
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) { delete c; return DCPP_ERR_CUDA; }
  if (prop.major != 10) {
    delete c;
    return DCPP_ERR_UNSUPPORTED;  // built for sm_100a only
  }
  c->num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->own_stream, cudaStreamNonBlocking) != cudaSuccess) { delete c; return DCPP_ERR_CUDA; }
  c->stream = c->own_stream;
  if (cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess || cudaMemset(c->d_err, 0, sizeof(int)) != cudaSuccess) {
    cudaStreamDestroy(c->own_stream);
    delete c;
    return DCPP_ERR_CUDA;
  }
  *out_ctx = c;
  return DCPP_OK;
}

dcpp_status dcpp_destroy(dcpp_ctx* ctx) {
  if (!ctx) return DCPP_ERR_INVALID_ARG;
  cudaSetDevice(ctx->device);
  if (ctx->comm) {
    try { dcpp::Nccl::get().CommDestroy(ctx->comm); } catch (...) {}
  }
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->scratch) cudaFree(ctx->scratch);
  if (ctx->split_ws) cudaFree(ctx->split_ws);
  if (ctx->d_err) cudaFree(ctx->d_err);
  if (ctx->own_stream) cudaStreamDestroy(ctx->own_stream);
  delete ctx;
  return DCPP_OK;
}

const char* dcpp_last_error(const dcpp_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "null context"; }

dcpp_status dcpp_set_stream(dcpp_ctx* ctx, void* s) {
  return guarded(ctx, "dcpp_set_stream", [&] {
    ctx->stream = s ? static_cast<cudaStream_t>(s) : ctx->own_stream;
  });
}

dcpp_status dcpp_synchronize(dcpp_ctx* ctx) {
  return guarded(ctx, "dcpp_synchronize", [&] { ctx->check_device_error(); });
}

dcpp_status dcpp_alloc(dcpp_ctx* ctx, size_t bytes, void** d_out) {
  return guarded(ctx, "dcpp_alloc", [&] {
    if (!d_out) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_alloc: null output");
    *d_out = nullptr;
    if (cudaMalloc(d_out, bytes ? bytes : 1) != cudaSuccess) {
      cudaGetLastError();
      dcpp::fail(DCPP_ERR_OOM, "cudaMalloc of " + std::to_string(bytes) + " bytes failed");
    }
  });
}

dcpp_status dcpp_free(dcpp_ctx* ctx, void* p) {
  return guarded(ctx, "dcpp_free", [&] { dcpp::cuda_check(cudaFree(p), "cudaFree"); });
}

dcpp_status dcpp_memcpy(dcpp_ctx* ctx, void* dst, const void* src, size_t bytes) {
  return guarded(ctx, "dcpp_memcpy", [&] {
    dcpp::cuda_check(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, ctx->stream), "cudaMemcpyAsync");
    dcpp::cuda_check(cudaStreamSynchronize(ctx->stream), "cudaStreamSynchronize");
  });
}

dcpp_status dcpp_row_bytes(int type, int64_t n, size_t* out) {
  if (!out || n < 0) return DCPP_ERR_INVALID_ARG;
  try {
    *out = dcpp::row_bytes_of(type, n);
    return DCPP_OK;
  } catch (const Error& e) {
    return e.status;
  }
}

dcpp_status dcpp_inject_fault(dcpp_ctx* ctx, const char* name, int nth) {
  if (!ctx) return DCPP_ERR_INVALID_ARG;
  if (!name || nth <= 0) {
    ctx->fault_name.clear();
    ctx->fault_countdown = 0;
  } else {
    ctx->fault_name = name;
    ctx->fault_countdown = nth;
  }
  return DCPP_OK;
}

dcpp_status dcpp_dequant(dcpp_ctx* ctx, int type, const void* blocks, int64_t n, float* out) {
  return guarded(ctx, "dcpp_dequant", [&] {
    if (!blocks || !out || n < 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_dequant: bad argument");
    (void)dcpp::row_bytes_of(type, n);
    dcpp::cuda_check(dcpp::launch_dequant_f32(type, blocks, n, out, ctx->stream), "dequant");
  });
}

dcpp_status dcpp_dequant_bf16(dcpp_ctx* ctx, int type, const void* blocks, int64_t n, uint16_t* out) {
  return guarded(ctx, "dcpp_dequant_bf16", [&] {
    if (!blocks || !out || n < 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_dequant_bf16: bad argument");
    (void)dcpp::row_bytes_of(type, n);
    dcpp::cuda_check(dcpp::launch_dequant_bf16(type, blocks, n, out, ctx->stream), "dequant");
  });
}

dcpp_status dcpp_f32_to_bf16(dcpp_ctx* ctx, const float* in, int64_t n, uint16_t* out) {
  return guarded(ctx, "dcpp_f32_to_bf16", [&] {
    if (!in || !out || n < 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_f32_to_bf16: bad argument");
    dcpp::cuda_check(dcpp::launch_f32_to_bf16(in, n, out, ctx->stream), "f32_to_bf16");
  });
}

dcpp_status dcpp_gemm(dcpp_ctx* ctx, int wtype, const void* w, int64_t N, int64_t K, const uint16_t* x, int64_t M,
                      float* y) {
  return guarded(ctx, "dcpp_gemm", [&] {
    if (!w || !x || !y) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_gemm: null pointer");
    dcpp::gemm_op(*ctx, wtype, w, N, K, x, M, y);
  });
}

dcpp_status dcpp_set_gemm_kernel(dcpp_ctx* ctx, int kind) {
  return guarded(ctx, "dcpp_set_gemm_kernel", [&] {
    if (kind < 0 || kind > 2) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_set_gemm_kernel: 0 auto, 1 single-SM, 2 CTA pairs");
    ctx->gemm_kernel = kind;
  });
}

dcpp_status dcpp_set_attention_kernel(dcpp_ctx* ctx, int kind) {
  return guarded(ctx, "dcpp_set_attention_kernel", [&] {
    if (kind < 0 || kind > 2) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_set_attention_kernel: 0 auto, 1 one tile, 2 two tiles");
    ctx->attn_kernel = kind;
  });
}

dcpp_status dcpp_set_wait_timeout(dcpp_ctx* ctx, double seconds) {
  return guarded(ctx, "dcpp_set_wait_timeout", [&] {
    if (!(seconds == 0.0 || (seconds >= 1e-3 && seconds <= 60.0)))
      dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_set_wait_timeout: 0 (default) or 0.001 .. 60 seconds");
    ctx->wait_timeout_ns = static_cast<uint64_t>(seconds * 1e9);
  });
}

dcpp_status dcpp_tp_barrier_selftest(dcpp_ctx* ctx, int nranks, uint32_t arrived_mask) {
  return guarded(ctx, "dcpp_tp_barrier_selftest", [&] {
    if (nranks < 1 || nranks > 8) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_tp_barrier_selftest: nranks must be 1..8");
    // One 32-word flag array per emulated rank, then the epoch counter.
    uint32_t* buf = nullptr;
    const size_t words = 32 * 8 + 32;
    dcpp::cuda_check(cudaMalloc(&buf, words * 4), "dcpp_tp_barrier_selftest: cudaMalloc");
    std::vector<uint32_t> init(words, 0u);
    // Rank j that "arrived" has already stored epoch 1 into rank 0's array.
    for (int j = 1; j < nranks; ++j)
      if (arrived_mask & (1u << j)) init[j] = 1u;
    dcpp::TpBarrierArgs a{};
    for (int j = 0; j < nranks; ++j) a.flags[j] = buf + 32 * j;
    a.epoch = buf + 32 * 8;
    a.err = ctx->d_err;
    a.rank = 0;
    a.nranks = nranks;
    a.timeout_ns = ctx->wait_timeout_ns;
    cudaError_t e = cudaMemcpyAsync(buf, init.data(), words * 4, cudaMemcpyHostToDevice, ctx->stream);
    if (e == cudaSuccess) e = dcpp::launch_tp_barrier(a, ctx->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    cudaFree(buf);
    dcpp::cuda_check(e, "dcpp_tp_barrier_selftest");
    ctx->check_device_error();
  });
}

dcpp_status dcpp_packed_bytes(int type, int64_t N, int64_t K, size_t* out) {
  if (!out || N <= 0 || K <= 0) return DCPP_ERR_INVALID_ARG;
  if ((type != DCPP_TYPE_Q4_K && type != DCPP_TYPE_Q8_0) || (type == DCPP_TYPE_Q4_K && K % 256) || K % 64)
    return DCPP_ERR_UNSUPPORTED;
  *out = dcpp::packed_bytes(type, N, K);
  return DCPP_OK;
}

dcpp_status dcpp_pack_weight(dcpp_ctx* ctx, int type, const void* raw, int64_t N, int64_t K, void* out) {
  return guarded(ctx, "dcpp_pack_weight", [&] {
    if (!raw || !out || N <= 0 || K <= 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_pack_weight: bad argument");
    if ((type != DCPP_TYPE_Q4_K && type != DCPP_TYPE_Q8_0) || (type == DCPP_TYPE_Q4_K && K % 256) || K % 64)
      dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_pack_weight: Q4_K (K % 256 == 0) or Q8_0 (K % 64 == 0) only");
    dcpp::cuda_check(dcpp::launch_pack_weight(type, raw, N, K, out, ctx->stream), "pack weight");
  });
}

dcpp_status dcpp_gemm_packed(dcpp_ctx* ctx, int wtype, const void* packed, int64_t N, int64_t K, const uint16_t* x,
                             int64_t M, float* y) {
  return guarded(ctx, "dcpp_gemm_packed", [&] {
    if (!packed || !x || !y || N <= 0 || K <= 0 || M <= 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_gemm_packed: bad argument");
    if ((wtype != DCPP_TYPE_Q4_K && wtype != DCPP_TYPE_Q8_0) || K % 64)
      dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm_packed: packed Q4_K / Q8_0 weights with K % 64 == 0 only");
    if (M > INT32_MAX / 2 || N > INT32_MAX / 2) dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm_packed: size too large");
    CUtensorMap ta;
    dcpp::cuda_check(dcpp::make_tmap_bf16(&ta, x, K, M, K, dcpp::kGemmBM), "tensor map (x)");
    dcpp::GemmArgs a{};
    a.N = static_cast<int32_t>(N);
    a.K = static_cast<int32_t>(K);
    a.n_groups = 1;
    a.groups[0].rows = static_cast<int32_t>(M);
    a.ep.mode = dcpp::kEpiF32;
    a.ep.out_f32 = y;
    a.ep.ld_out = N;
    a.qb[0].packed = packed;
    a.qb[1].packed = packed;
    a.err = ctx->d_err;
    const bool pair = ctx->use_pair(M, /*fused_dequant=*/true);
    dcpp::gemm_finalize_groups(a, pair ? 256 : dcpp::kGemmBM);
    const int bsrc = wtype == DCPP_TYPE_Q4_K ? dcpp::kBSrcQ4_K : dcpp::kBSrcQ8_0;
    if (pair)
      dcpp::cuda_check(dcpp::launch_gemm_pair(ta, ta, ta, a, bsrc, ctx->num_sms, ctx->stream), "launch fused gemm (pair)");
    else
      dcpp::cuda_check(dcpp::launch_gemm(ta, ta, ta, a, bsrc, ctx->num_sms, ctx->stream), "launch fused gemm");
  });
}

dcpp_status dcpp_layernorm_mod(dcpp_ctx* ctx, const float* x, int64_t rows, int64_t D, const float* shift,
                               const float* scale, float eps, uint16_t* y) {
  return guarded(ctx, "dcpp_layernorm_mod", [&] {
    if (!x || !y || rows < 0 || D <= 0) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_layernorm_mod: bad argument");
    if (D % 4 || D > 8192) dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_layernorm_mod: D must be a multiple of 4, <= 8192");
    if (rows > INT32_MAX) dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_layernorm_mod: too many rows");
    dcpp::NormArgs a{};
    a.x = x;
    a.y = y;
    a.ld_x = D;
    a.ld_y = D;
    a.D = static_cast<int32_t>(D);
    a.eps = eps;
    a.n_segments = 1;
    a.seg[0] = {0, 0, static_cast<int32_t>(rows), shift, scale};
    dcpp::cuda_check(dcpp::launch_layernorm_mod(a, ctx->stream), "layernorm_mod");
  });
}

dcpp_status dcpp_attention(dcpp_ctx* ctx, const uint16_t* qkv, int64_t B, int64_t S, int64_t H, int64_t head_dim,
                           const float* norm_q, const float* norm_k, float eps, const int32_t* ids, int n_axes,
                           const int64_t* axes_dims, float theta, uint16_t* out) {
  return guarded(ctx, "dcpp_attention", [&] {
    if (!qkv || !out || !ids || !norm_q || !norm_k || !axes_dims || B <= 0 || S <= 0 || H <= 0)
      dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_attention: bad argument");
    if (head_dim != 128) dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_attention: head_dim must be 128");
    if (n_axes < 1 || n_axes > 8) dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_attention: 1..8 rope axes");
    int32_t dims[8];
    int64_t tot = 0;
    for (int i = 0; i < n_axes; ++i) {
      dims[i] = static_cast<int32_t>(axes_dims[i]);
      tot += axes_dims[i];
    }
    if (tot != head_dim) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_attention: axes dims must sum to head_dim");
    if (B * H > 65535 || S > (1 << 24)) dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_attention: size too large");
    const int64_t sp = dcpp::attn_vt_stride(S);
    const size_t qk_elems = static_cast<size_t>(B * H * S * 128);
    const size_t vt_elems = static_cast<size_t>(B * H * 128 * sp);
    const size_t rope_off = ((2 * qk_elems + vt_elems) * 2 + 255) & ~size_t(255);
    const size_t need = rope_off + static_cast<size_t>(S) * 64 * sizeof(float2);
    uint8_t* s = static_cast<uint8_t*>(ctx->ensure_scratch(need));
    auto* q = reinterpret_cast<uint16_t*>(s);
    auto* k = q + qk_elems;
    auto* vt = k + qk_elems;
    auto* rope = reinterpret_cast<float2*>(s + rope_off);
    // The V^T padding columns [S, sp) must hold finite values (zeros).
    dcpp::cuda_check(cudaMemsetAsync(vt, 0, vt_elems * 2, ctx->stream), "memset vt");
    dcpp::cuda_check(dcpp::launch_rope_table(ids, S, n_axes, dims, theta, rope, ctx->stream), "rope table");
    dcpp::cuda_check(dcpp::launch_qk_norm_rope(qkv, B, S, H, norm_q, norm_k, eps, rope, q, k, vt, sp, ctx->stream),
                     "qk norm rope");
    dcpp::AttnTcMaps maps;
    dcpp::cuda_check(dcpp::make_attn_maps(&maps, q, k, vt, static_cast<int>(B), static_cast<int>(H),
                                          static_cast<int>(S)),
                     "attention tensor maps");
    dcpp::AttnTcArgs a{};
    a.o = out;
    a.ld_o = H * 128;
    a.B = static_cast<int32_t>(B);
    a.H = static_cast<int32_t>(H);
    a.S = static_cast<int32_t>(S);
    a.scale = 1.0f / sqrtf(128.0f);
    a.err = ctx->d_err;
    a.kernel = ctx->attn_kernel;
    dcpp::cuda_check(dcpp::launch_attention_tc(maps, a, ctx->stream), "attention");
  });
}

dcpp_status dcpp_tp_get_unique_id(void* id_out) {
  if (!id_out) return DCPP_ERR_INVALID_ARG;
  try {
    auto& n = dcpp::Nccl::get();
    dcpp::Nccl::UniqueId id;
    if (n.GetUniqueId(&id) != 0) return DCPP_ERR_NCCL;
    memcpy(id_out, &id, sizeof(id));
    return DCPP_OK;
  } catch (const Error& e) {
    return e.status;
  }
}

dcpp_status dcpp_tp_init(dcpp_ctx* ctx, int rank, int nranks, const void* nccl_id) {
  return guarded(ctx, "dcpp_tp_init", [&] {
    if (!nccl_id || nranks < 1 || rank < 0 || rank >= nranks) dcpp::fail(DCPP_ERR_INVALID_ARG, "dcpp_tp_init: bad rank");
    auto& n = dcpp::Nccl::get();
    dcpp::Nccl::UniqueId id;
    memcpy(&id, nccl_id, sizeof(id));
    dcpp::Nccl::Comm comm = nullptr;
    int r = n.CommInitRank(&comm, nranks, id, rank);
    if (r != 0) dcpp::fail(DCPP_ERR_NCCL, std::string("ncclCommInitRank: ") + n.GetErrorString(r));
    ctx->comm = comm;
    ctx->rank = rank;
    ctx->nranks = nranks;
  });
}

dcpp_status dcpp_allreduce(dcpp_ctx* ctx, void* buf, int64_t count, int dtype) {
  return guarded(ctx, "dcpp_allreduce", [&] {
    if (!ctx->comm) dcpp::fail(DCPP_ERR_STATE, "dcpp_allreduce: no TP group (call dcpp_tp_init)");
    int nd;
    if (dtype == DCPP_TYPE_F32) nd = 7;        // ncclFloat32
    else if (dtype == DCPP_TYPE_BF16) nd = 9;  // ncclBfloat16
    else dcpp::fail(DCPP_ERR_UNSUPPORTED, "dcpp_allreduce: F32 or BF16 only");
    auto& n = dcpp::Nccl::get();
    int r = n.AllReduce(buf, buf, static_cast<size_t>(count), nd, /*ncclSum*/ 0, ctx->comm, ctx->stream);
    if (r != 0) dcpp::fail(DCPP_ERR_NCCL, std::string("ncclAllReduce: ") + n.GetErrorString(r));
  });
}

}  // extern "C"
