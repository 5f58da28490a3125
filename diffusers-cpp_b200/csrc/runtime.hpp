// Host runtime shared by the C ABI and the C++ model: the context (device,
// stream, error state, fault injection, scratch), checked CUDA calls and
// the NCCL binding loaded at run time.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <stdexcept>
#include <string>

#include "../../include/dcpp.h"

namespace dcpp {

// Thrown inside the library, turned into a status at the C boundary.
struct Error : std::runtime_error {
  dcpp_status status;
  Error(dcpp_status s, const std::string& msg) : std::runtime_error(msg), status(s) {}
};

[[noreturn]] inline void fail(dcpp_status s, const std::string& msg) { throw Error(s, msg); }

inline void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) fail(DCPP_ERR_CUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

// Minimal NCCL ABI (types and the functions the library uses), resolved
// with dlopen("libnccl.so.2") so that the library has no link-time NCCL
// dependency and shares the NCCL that the process already loaded.
struct Nccl {
  using Comm = void*;
  struct UniqueId { char internal[DCPP_NCCL_ID_BYTES]; };
  int (*GetUniqueId)(UniqueId*) = nullptr;
  int (*CommInitRank)(Comm*, int, UniqueId, int) = nullptr;
  int (*CommDestroy)(Comm) = nullptr;
  int (*CommAbort)(Comm) = nullptr;
  int (*AllReduce)(const void*, void*, size_t, int, int, Comm, cudaStream_t) = nullptr;
  int (*AllGather)(const void*, void*, size_t, int, Comm, cudaStream_t) = nullptr;
  const char* (*GetErrorString)(int) = nullptr;
  bool loaded = false;
  static Nccl& get();  // loads on first use; throws DCPP_ERR_NCCL when missing
};

struct Ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  cudaStream_t own_stream = nullptr;
  std::string last_error = "";
  int* d_err = nullptr;  // device error word written by bounded waits
  // Fault injection (host side only).
  std::string fault_name;
  int fault_countdown = 0;
  // Scratch for the op-level GEMM (bf16 weights) and staging, and the K-split
  // partials of the op-level GEMM.
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  void* split_ws = nullptr;
  size_t split_ws_bytes = 0;
  // GEMM kernel choice: 0 auto, 1 single-SM 128 x 256 tiles, 2 CTA-pair
  // 256 x 256 tiles.  Auto takes CTA pairs for bf16 weights and >= 256 rows,
  // and the single-SM kernel for fused dequantisation (measured faster: the
  // pair kernel is bound by shared-memory bandwidth once B is written there).
  int gemm_kernel = 0;
  int attn_kernel = 0;  // 0 auto, 1 one query tile per CTA, 2 two tiles
  // Limit of the cross-GPU barrier waits of plans prepared afterwards
  // (dcpp_set_wait_timeout); 0 = the library default of 1 s.
  uint64_t wait_timeout_ns = 0;
  bool use_pair(int64_t rows, bool fused_dequant = false) const {
    return gemm_kernel == 2 || (gemm_kernel == 0 && rows >= 256 && !fused_dequant);
  }
  // Tensor parallelism.
  Nccl::Comm comm = nullptr;
  int rank = 0;
  int nranks = 1;

  void maybe_inject(const char* entry);
  void* ensure_scratch(size_t bytes);
  void* ensure_split_ws(size_t bytes);
  // Read and clear the device error word (synchronises the stream).
  void check_device_error();
};

const char* device_error_name(int code);

// A device buffer of the same size on every rank of the context's TP group,
// with every peer's copy mapped into this process (CUDA IPC; the handles are
// exchanged with an NCCL all-gather).  open() and close() are collective.
// peer[j] is rank j's buffer (peer[rank] == local); kernels of this library
// store into peers' buffers over NVLink with plain loads and stores.
struct PeerBuffer {
  uint8_t* local = nullptr;
  size_t bytes = 0;
  uint8_t* peer[8] = {};
  void open(Ctx& ctx, size_t bytes);
  void close(Ctx& ctx);
};

}  // namespace dcpp

struct dcpp_ctx : dcpp::Ctx {};
