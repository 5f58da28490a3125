// Allocation-free variant of the GEMM entry point (dcpp_gemm_noalloc).
//
// dcpp_gemm expands a quantised weight to bf16 in a scratch buffer that the
// context grows with cudaMalloc.  Some callers cannot allow that: a host
// framework that owns every device allocation through its own pool (as ggml's
// backend buffers do), a caller in the middle of recording work that must not
// trigger a device-wide synchronising call such as cudaMalloc / cudaFree, or
// a deployment with a fixed memory budget checked up front.  For them this
// file keeps the scratch in a fixed device array that is part of the loaded
// library: nothing is allocated per call.
//
// The scratch is kNoAllocScratchBytes (32 MiB) per GPU that loads the library,
// held until the process exits.  Weights larger than that are expanded and
// multiplied in row chunks that fit it, so the only size limit is
// K <= 65536 (one chunk of 256 output rows must fit).
//
// The array is shared by every call on a device and keeps the last call's
// contents; each call fully overwrites the part it reads, so nothing has to
// start at zero.  Calls whose GPU work overlaps (two streams, or two
// contexts on one device) race on the array and must be serialised by the
// caller.
#include <cuda.h>

#include <mutex>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "runtime.hpp"

namespace dcpp {

size_t row_bytes_of(int type, int64_t n);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;

// Device-side scratch.  In host code this name is only a stand-in for the
// symbol: its device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

// Device address of the scratch, looked up once per CUDA context: keyed on
// the current context (not the device id), so a context that the host
// destroys and re-creates (cudaDeviceReset, primary-context release) gets
// its own lookup instead of a stale address.
std::mutex g_scratch_mu;
struct ScratchAddr {
  CUcontext cu_ctx;
  void* addr;
};
std::vector<ScratchAddr> g_scratch_addrs;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CUcontext current_cu_context() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<CtxGetCurrentFn>(p);
  }();
  if (!fn) fail(DCPP_ERR_CUDA, "dcpp_gemm_noalloc: cuCtxGetCurrent is unavailable");
  CUcontext c = nullptr;
  if (fn(&c) != CUDA_SUCCESS || !c) fail(DCPP_ERR_CUDA, "dcpp_gemm_noalloc: no current CUDA context");
  return c;
}

// Device address of the scratch in the current context (the caller made
// the context's device current and the runtime initialised it).  The first
// call in a context looks it up with cudaGetSymbolAddress; later calls
// reuse it.
void* noalloc_scratch() {
  const CUcontext cu = current_cu_context();
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  for (const auto& e : g_scratch_addrs)
    if (e.cu_ctx == cu) return e.addr;
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess || !p)
    fail(DCPP_ERR_CUDA, std::string("dcpp_gemm_noalloc: cudaGetSymbolAddress failed: ") + cudaGetErrorString(e));
  g_scratch_addrs.push_back({cu, p});
  return p;
}

void gemm_chunk(Ctx& c, const uint16_t* wb, int64_t rows, int64_t K, const uint16_t* x, int64_t M, float* y,
                int64_t ld_y) {
  CUtensorMap ta, tb;
  cuda_check(make_tmap_bf16(&ta, x, K, M, K, kGemmBM), "dcpp_gemm_noalloc: tensor map (x)");
  cuda_check(make_tmap_bf16(&tb, wb, K, rows, K, kGemmBN), "dcpp_gemm_noalloc: tensor map (W)");
  GemmArgs a{};
  a.N = static_cast<int32_t>(rows);
  a.K = static_cast<int32_t>(K);
  a.n_groups = 1;
  a.groups[0].rows = static_cast<int32_t>(M);
  a.ep.mode = kEpiF32;
  a.ep.out_f32 = y;
  a.ep.ld_out = ld_y;
  a.err = c.d_err;
  gemm_finalize_groups(a);
  cuda_check(launch_gemm(ta, tb, tb, a, kBSrcBf16, c.num_sms, c.stream), "dcpp_gemm_noalloc: gemm");
}

void gemm_noalloc(Ctx& c, int wtype, const void* w, int64_t N, int64_t K, const uint16_t* x, int64_t M, float* y) {
  if (!w || !x || !y) fail(DCPP_ERR_INVALID_ARG, "dcpp_gemm_noalloc: null pointer");
  if (N <= 0 || K <= 0 || M <= 0) fail(DCPP_ERR_INVALID_ARG, "dcpp_gemm_noalloc: sizes must be positive");
  if (K % 8) fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm_noalloc: K must be a multiple of 8");
  if (M > INT32_MAX / 2 || N > INT32_MAX / 2) fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm_noalloc: size too large");
  const size_t rb = row_bytes_of(wtype, K);
  if (wtype == kTypeBF16) {  // no expansion needed
    gemm_chunk(c, static_cast<const uint16_t*>(w), N, K, x, M, y, N);
    return;
  }
  // Output rows per chunk: as many 256-row tiles as fit the scratch.
  const int64_t max_rows = static_cast<int64_t>(kNoAllocScratchBytes / (static_cast<size_t>(K) * 2)) / kGemmBN * kGemmBN;
  if (max_rows < kGemmBN)
    fail(DCPP_ERR_UNSUPPORTED, "dcpp_gemm_noalloc: K = " + std::to_string(K) +
                                   " exceeds the allocation-free scratch (32 MiB holds 256 bf16 rows of K <= 65536)");
  uint16_t* scratch = static_cast<uint16_t*>(noalloc_scratch());
  const uint8_t* wbytes = static_cast<const uint8_t*>(w);
  for (int64_t n0 = 0; n0 < N; n0 += max_rows) {
    const int64_t rows = std::min(max_rows, N - n0);
    cuda_check(launch_dequant_bf16(wtype, wbytes + static_cast<size_t>(n0) * rb, rows * K, scratch, c.stream),
               "dcpp_gemm_noalloc: dequant");
    gemm_chunk(c, scratch, rows, K, x, M, y + n0, N);
  }
}

}  // namespace
}  // namespace dcpp

extern "C" dcpp_status dcpp_gemm_noalloc(dcpp_ctx* ctx, int wtype, const void* d_w, int64_t N, int64_t K,
                                         const uint16_t* d_x, int64_t M, float* d_y) {
  if (!ctx) return DCPP_ERR_INVALID_ARG;
  try {
    ctx->maybe_inject("dcpp_gemm_noalloc");
    cudaSetDevice(ctx->device);
    dcpp::gemm_noalloc(*ctx, wtype, d_w, N, K, d_x, M, d_y);
    return DCPP_OK;
  } catch (const dcpp::Error& e) {
    ctx->last_error = e.what();
    return e.status;
  } catch (const std::exception& e) {
    ctx->last_error = e.what();
    return DCPP_ERR_INVALID_ARG;
  }
}
