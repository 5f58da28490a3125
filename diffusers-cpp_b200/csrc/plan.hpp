// Execution plans shared by the models: a step is a fixed list of ops
// (kernel launches, stream records / waits) built once per problem size,
// issued on the context's stream plus one side stream, optionally captured
// into a CUDA graph, and optionally bracketed by CUDA events per op for
// profiling.  Also the device-resident parameter types and the host-side
// helpers the model loaders share (ggml block sizes, host dequantisation,
// a flat config.json reader).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include <functional>
#include <map>
#include <set>
#include <string>
#include <vector>

#include "gemm.cuh"
#include "kernels.cuh"
#include "runtime.hpp"

namespace dcpp {

// A weight matrix [rows, cols] of one ggml type, as raw GGUF rows on the
// device, assembled from one or more named parts.
struct DevWeight {
  std::string name;
  int type = -1;
  int64_t rows = 0;
  int64_t cols = 0;
  size_t row_bytes = 0;
  uint8_t* data = nullptr;             // device, raw GGUF rows (null once packed)
  uint8_t* packed = nullptr;           // device, fused-dequant stage layout (block projections)
  bool pack = false;                   // a block projection: pack when quantised
  bool on_host = false;                // host-only model: assembled rows kept in `staging`
  std::vector<uint8_t> staging;        // host, until all parts arrived
  std::set<std::string> need;          // part names still missing
  bool ready() const { return (data != nullptr || packed != nullptr || on_host) && need.empty(); }
};

// An f32 vector parameter (norm weights).
struct DevVector {
  std::string name;
  int64_t n = 0;
  float* data = nullptr;
  std::vector<float> host;  // host-only model
  bool set = false;
};

size_t row_bytes_of(int type, int64_t n);
int64_t block_size_of(int type);
size_t block_bytes_of(int type);
uint16_t host_f32_to_bf16(float f);
// Dequantise one GGUF row of n weights to f32 (the gguf-py arithmetic).
void host_dequant_row(int type, const uint8_t* src, int64_t n, float* out);
bool is_gemm_type(int t);
std::string shape_str(const std::vector<int64_t>& s);
// A flat JSON object (config.json) as key -> raw value text.
std::map<std::string, std::string> read_json_object(const std::string& path);
std::vector<int64_t> parse_int_list(const std::string& v);
// Upload an f32 / f16 / bf16 vector parameter as f32 (checks shape and size).
void set_vector_param(DevVector& v, int type, const std::vector<int64_t>& shape, const void* data, size_t nbytes,
                      bool host_only);

class StepPlanner {
 public:
  enum ProfileKind { kOpGemm = 0, kOpAttention = 1, kOpNorm = 2, kOpGemv = 3, kOpDequant = 4, kOpOther = 5,
                     kOpAllreduce = 6, kOpKinds = 7 };
  explicit StepPlanner(Ctx& ctx) : ctx_(ctx) {}
  virtual ~StepPlanner();
  // Per-kind milliseconds / FLOPs / launches of the last executed step
  // (profiling must have been on when the plan was built).
  void profile(int kind, double* ms, double* flops, int64_t* launches);
  int64_t launches_per_step() const { return launches_per_step_; }

 protected:
  struct Op {
    std::function<void(cudaStream_t)> fn;
    int launches;
    int kind = kOpOther;   // ProfileKind
    double flops = 0.0;    // algorithmic FLOPs of the op
    std::string tag;       // what the op is (profile dumps)
    int stream = 0;        // 0: the context's stream, 1: the side stream, 2: the expansion stream
    bool timed = true;     // false for stream records / waits (not profiled)
  };

  // Start / finish building one op list: the side streams join the list at
  // its start and rejoin the main stream at its end (a captured graph must
  // end on its origin stream).
  void begin_ops(std::vector<Op>& ops);
  void end_ops();
  // Allocate the bf16 expansion scratch (two pairs of s0 / s1 elements).
  void alloc_expansion_scratch(const std::function<void*(size_t)>& alloc, size_t s0, size_t s1);
  // Block-ahead weight expansion: two sets of `elems` bf16 elements.
  void alloc_prefetch_scratch(const std::function<void*(size_t)>& alloc, size_t elems);
  // Expand the quantised (raw, not packed) weights of `ws` into prefetch set
  // `set` on the expansion stream, starting when the main stream reaches
  // this point of the plan; later GEMMs reading these weights use the
  // expansion and wait for it.  The caller guarantees that every GEMM that
  // read the set's previous contents precedes this point on the main stream.
  void add_prefetch(const std::vector<const DevWeight*>& ws, int set);
  cudaStream_t op_stream(int i) const { return i == 0 ? ctx_.stream : (i == 1 ? side_ : side2_); }
  void release_plan_events();
  void run_ops(std::vector<Op>& ops, cudaGraphExec_t* graph);

  void add_gemm(const std::string& tag, const uint16_t* a, int64_t lda, int64_t K, const DevWeight* w0,
                const DevWeight* w1, std::vector<GemmGroup> groups, const EpilogueArgs& ep, int64_t N);
  // The same GEMM launched once per row piece (weights expanded once);
  // before_piece(p) emits what must precede piece p.
  void add_gemm_pieces(const std::string& tag, const uint16_t* a, int64_t lda, int64_t K, const DevWeight* w0,
                       const DevWeight* w1, const std::vector<std::vector<GemmGroup>>& pieces, const EpilogueArgs& ep,
                       int64_t N, const std::function<void(int)>& before_piece);
  void add_norm(const NormArgs& a, int stream = 0);
  // Arrival waits for the next GEMM built (consumed by it): its CTA-pair
  // kernel waits for the A rows other GPUs push (GemmArgs::ag_*) and walks
  // its tiles M tile by M tile, in the order the rows arrive.
  // The overlapped all-gather the next GEMM runs (GemmArgs::ag_*): it
  // pushes this rank's granules of `a` and waits for the others'.
  struct AgWait {
    const uint32_t* flags = nullptr;
    const uint32_t* step = nullptr;
    int32_t site = 0, rank = 0, n = 0;
    int32_t rows = 0;
    int64_t ld = 0;
    const uint16_t* a = nullptr;
    uint16_t* a_peer[8] = {};
    uint32_t* flags_peer[8] = {};
    uint32_t* count = nullptr;
  };
  AgWait next_ag_{};
  void add_gemv(const DevWeight& w, const float* x, int batch, int act_in, int act_out, float* y);
  // Cross-stream dependencies inside a plan (graph edges when captured).
  cudaEvent_t plan_event();
  void add_record(cudaEvent_t e, int stream);
  void add_wait(cudaEvent_t e, int stream);

  Ctx& ctx_;
  bool use_graph_ = false;
  bool profiling_ = false;
  int64_t launches_per_step_ = 0;
  std::vector<Op>* building_ = nullptr;
  std::vector<Op>* last_ops_ = nullptr;
  std::vector<cudaEvent_t> ev_;  // 2 per op of the largest plan (profiling)
  // bf16 expansion of quantised GEMM weights: two pairs (first / second
  // weight of one launch), used alternately, so that the expansion of the
  // next projection runs on the side stream while the current GEMM computes.
  // Ring of expansion scratch pairs: a GEMM's weight expansion may start once
  // the GEMM that used its pair n_scratch_ expanding GEMMs back has finished.
  static constexpr int kMaxScratch = 3;
  int n_scratch_ = 2;
  uint16_t* wscratch_[kMaxScratch][2] = {};
  int scratch_pair_ = 0;
  cudaEvent_t scratch_free_[kMaxScratch] = {};  // last GEMM that read the pair (null: none yet)
  cudaEvent_t plan_start_ = nullptr;                   // recorded on the main stream first in a plan
  cudaStream_t side_ = nullptr;
  cudaStream_t side2_ = nullptr;  // block-ahead weight expansions
  struct Prefetched {
    uint16_t* dst;
    cudaEvent_t ready;
  };
  std::map<const DevWeight*, Prefetched> prefetched_;  // of the op list being built
  uint16_t* pf_scratch_[2] = {};
  size_t pf_scratch_elems_ = 0;
  std::vector<cudaEvent_t> plan_events_;
  // f32 partials of K-split GEMMs (shared by every split launch of the
  // model's plans, which run in order on one stream).
  float* split_ws_ = nullptr;
  size_t split_ws_bytes_ = 0;
  int64_t split_launches_ = 0;  // split launches in the current plans (the workspace may grow only at 0)
};

}  // namespace dcpp
