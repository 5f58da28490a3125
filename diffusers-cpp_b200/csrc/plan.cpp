// Shared execution-plan machinery and loader helpers (see plan.hpp).
#include "plan.hpp"

#include <cuda_fp16.h>
#include <string.h>

#include <algorithm>
#include <array>
#include <fstream>
#include <memory>
#include <sstream>

namespace dcpp {

namespace {

float host_f16_to_f32(const uint8_t* p) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// ---- a small JSON reader for diffusers config.json (flat object with
// numbers, booleans, null, strings and arrays of numbers).
struct Json {
  const std::string& s;
  size_t i = 0;
  explicit Json(const std::string& src) : s(src) {}
  void ws() {
    while (i < s.size() && isspace(static_cast<unsigned char>(s[i]))) ++i;
  }
  [[noreturn]] void bad() { fail(DCPP_ERR_INVALID_ARG, "config json: parse error at offset " + std::to_string(i)); }
  std::string str() {
    ws();
    if (i >= s.size() || s[i] != '"') bad();
    ++i;
    std::string r;
    while (i < s.size() && s[i] != '"') {
      if (s[i] == '\\' && i + 1 < s.size()) ++i;
      r += s[i++];
    }
    if (i >= s.size()) bad();
    ++i;
    return r;
  }
  // Returns a value as text: number, true/false/null, "string", or [a,b,..].
  std::string value() {
    ws();
    if (i >= s.size()) bad();
    if (s[i] == '"') return "\"" + str() + "\"";
    if (s[i] == '[' || s[i] == '{') {
      char open = s[i], close = open == '[' ? ']' : '}';
      int depth = 0;
      size_t st = i;
      bool in_str = false;
      for (; i < s.size(); ++i) {
        char c = s[i];
        if (in_str) {
          if (c == '\\') ++i;
          else if (c == '"') in_str = false;
          continue;
        }
        if (c == '"') in_str = true;
        else if (c == open) ++depth;
        else if (c == close && --depth == 0) { ++i; return s.substr(st, i - st); }
      }
      bad();
    }
    size_t st = i;
    while (i < s.size() && s[i] != ',' && s[i] != '}' && s[i] != ']' && !isspace(static_cast<unsigned char>(s[i]))) ++i;
    return s.substr(st, i - st);
  }
  std::map<std::string, std::string> object() {
    std::map<std::string, std::string> m;
    ws();
    if (i >= s.size() || s[i] != '{') bad();
    ++i;
    ws();
    if (i < s.size() && s[i] == '}') { ++i; return m; }
    for (;;) {
      std::string k = str();
      ws();
      if (i >= s.size() || s[i] != ':') bad();
      ++i;
      m[k] = value();
      ws();
      if (i < s.size() && s[i] == ',') { ++i; continue; }
      if (i < s.size() && s[i] == '}') { ++i; break; }
      bad();
    }
    return m;
  }
};

}  // namespace

int64_t block_size_of(int type) {
  if (type == kTypeQ8_0) return 32;
  if (type == kTypeQ4_K) return 256;
  return 1;
}
size_t block_bytes_of(int type) {
  switch (type) {
    case kTypeQ8_0: return 34;
    case kTypeQ4_K: return 144;
    case kTypeF32: return 4;
    default: return 2;
  }
}
uint16_t host_f32_to_bf16(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  if ((b & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((b >> 16) | 0x40);  // quiet NaN
  b += 0x7FFFu + ((b >> 16) & 1u);  // round to nearest even
  return static_cast<uint16_t>(b >> 16);
}


// Dequantise one GGUF row of n weights to f32 (the gguf-py arithmetic: Q8_0
// d * q; Q4_K (d * sc) * q - dmin * m), for load-time expansion only.
void host_dequant_row(int type, const uint8_t* src, int64_t n, float* out) {
  if (type == kTypeQ8_0) {
    for (int64_t b = 0; b < n / 32; ++b) {
      const uint8_t* blk = src + b * 34;
      const float d = host_f16_to_f32(blk);
      for (int i = 0; i < 32; ++i) out[b * 32 + i] = static_cast<float>(static_cast<int8_t>(blk[2 + i])) * d;
    }
  } else if (type == kTypeQ4_K) {
    for (int64_t b = 0; b < n / 256; ++b) {
      const uint8_t* blk = src + b * 144;
      const float d = host_f16_to_f32(blk), dmin = host_f16_to_f32(blk + 2);
      const uint8_t* s = blk + 4;
      for (int j = 0; j < 8; ++j) {
        int sc, m;
        if (j < 4) {
          sc = s[j] & 0x3F;
          m = s[j + 4] & 0x3F;
        } else {
          sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 2) & 0x30);
          m = (s[j + 4] >> 4) | ((s[j] >> 2) & 0x30);
        }
        const float ds = d * static_cast<float>(sc), dm = dmin * static_cast<float>(m);
        const uint8_t* qs = blk + 16 + (j / 2) * 32;
        for (int l = 0; l < 32; ++l) {
          const float q = static_cast<float>((qs[l] >> ((j & 1) * 4)) & 0x0F);
          const float prod = ds * q;
          out[b * 256 + j * 32 + l] = prod - dm;
        }
      }
    }
  } else {
    fail(DCPP_ERR_UNSUPPORTED, "host dequantisation: Q8_0 / Q4_K only");
  }
}

bool is_gemm_type(int t) {
  return t == kTypeQ8_0 || t == kTypeQ4_K || t == kTypeBF16 || t == kTypeF16 || t == kTypeF32;
}

std::string shape_str(const std::vector<int64_t>& s) {
  std::string r = "[";
  for (size_t i = 0; i < s.size(); ++i) r += (i ? ", " : "") + std::to_string(s[i]);
  return r + "]";
}

std::vector<int64_t> parse_int_list(const std::string& v) {
  std::vector<int64_t> r;
  std::string t;
  for (char c : v) {
    if (c == '[' || c == ']' || c == ',' || isspace(static_cast<unsigned char>(c))) {
      if (!t.empty()) { r.push_back(static_cast<int64_t>(std::stod(t))); t.clear(); }
    } else {
      t += c;
    }
  }
  if (!t.empty()) r.push_back(static_cast<int64_t>(std::stod(t)));
  return r;
}


std::map<std::string, std::string> read_json_object(const std::string& path) {
  std::ifstream f(path);
  if (!f.is_open()) fail(DCPP_ERR_NOT_FOUND, "Failed to open configuration file: " + path);
  std::stringstream ss;
  ss << f.rdbuf();
  std::string text = ss.str();
  Json j(text);
  return j.object();
}

void set_vector_param(DevVector& v, int type, const std::vector<int64_t>& shape, const void* data, size_t nbytes,
                      bool host_only) {
  if (shape.size() != 1 || shape[0] != v.n)
    fail(DCPP_ERR_INVALID_ARG, "Error while loading Tensor '" + v.name + "': Parameter shape mismatch: expected " +
                                   shape_str({v.n}) + ", got " + shape_str(shape));
  std::vector<float> host(static_cast<size_t>(v.n));
  const auto* u16 = static_cast<const uint16_t*>(data);
  if (type == kTypeF32) {
    if (nbytes != static_cast<size_t>(v.n) * 4) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + v.name + "': byte size mismatch");
    memcpy(host.data(), data, nbytes);
  } else if (type == kTypeBF16 || type == kTypeF16) {
    if (nbytes != static_cast<size_t>(v.n) * 2) fail(DCPP_ERR_INVALID_ARG, "Tensor '" + v.name + "': byte size mismatch");
    for (int64_t i = 0; i < v.n; ++i) {
      if (type == kTypeBF16) {
        uint32_t b = static_cast<uint32_t>(u16[i]) << 16;
        memcpy(&host[i], &b, 4);
      } else {
        host[i] = __half2float(__ushort_as_half(u16[i]));
      }
    }
  } else {
    fail(DCPP_ERR_UNSUPPORTED, "Tensor '" + v.name + "': norm weights must be F32, F16 or BF16");
  }
  if (host_only) {
    v.host.swap(host);
    v.set = true;
    return;
  }
  if (!v.data) cuda_check(cudaMalloc(&v.data, v.n * sizeof(float)), "alloc vector");
  cuda_check(cudaMemcpy(v.data, host.data(), v.n * sizeof(float), cudaMemcpyHostToDevice), "upload vector");
  v.set = true;
}

// ----------------------------------------------------------------- planner
StepPlanner::~StepPlanner() {
  if (split_ws_) cudaFree(split_ws_);
  for (auto e : ev_) cudaEventDestroy(e);
  release_plan_events();
  if (side_) cudaStreamDestroy(side_);
  if (side2_) cudaStreamDestroy(side2_);
}

void StepPlanner::release_plan_events() {
  for (auto e : plan_events_) cudaEventDestroy(e);
  plan_events_.clear();
  split_launches_ = 0;  // the plans that used the split workspace are gone
}

void StepPlanner::alloc_expansion_scratch(const std::function<void*(size_t)>& alloc, size_t s0, size_t s1) {
  if (const char* f = getenv("DCPP_EXPAND_AHEAD")) n_scratch_ = std::min(std::max(atoi(f), 2), kMaxScratch);
  for (int pi = 0; pi < n_scratch_; ++pi) {
    wscratch_[pi][0] = static_cast<uint16_t*>(alloc(std::max<size_t>(s0, 8) * 2));
    wscratch_[pi][1] = static_cast<uint16_t*>(alloc(std::max<size_t>(s1, 8) * 2));
  }
}

void StepPlanner::begin_ops(std::vector<Op>& ops) {
  if (!side_ || !side2_) {
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if (!side_) cuda_check(cudaStreamCreateWithPriority(&side_, cudaStreamNonBlocking, lo), "side stream");
    if (!side2_) cuda_check(cudaStreamCreateWithPriority(&side2_, cudaStreamNonBlocking, lo), "expansion stream");
  }
  building_ = &ops;
  scratch_pair_ = 0;
  for (auto& e : scratch_free_) e = nullptr;
  prefetched_.clear();
  plan_start_ = plan_event();
  add_record(plan_start_, 0);
  add_wait(plan_start_, 1);  // the side streams join the plan (and a capture) at its start
  add_wait(plan_start_, 2);
}

void StepPlanner::end_ops() {
  for (int st = 1; st <= 2; ++st) {
    cudaEvent_t side_done = plan_event();
    add_record(side_done, st);
    add_wait(side_done, 0);
  }
  prefetched_.clear();
  building_ = nullptr;
}

void StepPlanner::alloc_prefetch_scratch(const std::function<void*(size_t)>& alloc, size_t elems) {
  pf_scratch_elems_ = elems;
  for (int k = 0; k < 2; ++k) pf_scratch_[k] = elems ? static_cast<uint16_t*>(alloc(elems * 2)) : nullptr;
}

void StepPlanner::add_prefetch(const std::vector<const DevWeight*>& ws, int set) {
  std::vector<const DevWeight*> todo;
  size_t need = 0;
  for (const DevWeight* w : ws)
    if (w && w->data && !w->packed && w->type != kTypeBF16) {
      todo.push_back(w);
      need += (static_cast<size_t>(w->rows * w->cols) + 127) / 128 * 128;
    }
  if (todo.empty()) return;
  if (need > pf_scratch_elems_ || !pf_scratch_[set & 1])
    fail(DCPP_ERR_STATE, "internal: prefetch scratch too small for " + todo.front()->name);
  cudaEvent_t go = plan_event();
  add_record(go, 0);
  add_wait(go, 2);
  size_t off = 0;
  cudaEvent_t ready = plan_event();
  for (const DevWeight* w : todo) {
    uint16_t* dst = pf_scratch_[set & 1] + off;
    off += (static_cast<size_t>(w->rows * w->cols) + 127) / 128 * 128;
    Op o{[w, dst](cudaStream_t s) {
           cuda_check(launch_dequant_bf16(w->type, w->data, w->rows * w->cols, dst, s), "dequant");
         },
         1, kOpDequant, 0.0, "dequant (ahead) " + w->name};
    o.stream = 2;
    building_->push_back(o);
    prefetched_[w] = {dst, ready};
  }
  add_record(ready, 2);
}

cudaEvent_t StepPlanner::plan_event() {
  cudaEvent_t e;
  cuda_check(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "cudaEventCreate");
  plan_events_.push_back(e);
  return e;
}

void StepPlanner::add_record(cudaEvent_t e, int stream) {
  Op o{[e](cudaStream_t s) { cuda_check(cudaEventRecord(e, s), "event record"); }, 0, kOpOther, 0.0, "record"};
  o.stream = stream;
  o.timed = false;
  building_->push_back(o);
}

void StepPlanner::add_wait(cudaEvent_t e, int stream) {
  Op o{[e](cudaStream_t s) { cuda_check(cudaStreamWaitEvent(s, e, 0), "stream wait"); }, 0, kOpOther, 0.0, "wait"};
  o.stream = stream;
  o.timed = false;
  building_->push_back(o);
}

void StepPlanner::add_norm(const NormArgs& a, int stream) {
  Op o{[a](cudaStream_t s) { cuda_check(launch_layernorm_mod(a, s), "layernorm_mod"); }, 1, kOpNorm, 0.0,
       a.n_slots ? "layernorm+allgather" : "layernorm"};
  o.stream = stream;
  building_->push_back(o);
}

void StepPlanner::add_gemv(const DevWeight& w, const float* x, int batch, int act_in, int act_out, float* y) {
  const DevWeight* pw = &w;
  const int B = batch;
  building_->push_back({[pw, x, act_in, act_out, y, B](cudaStream_t s) {
                          cuda_check(launch_gemv(pw->type, pw->data, pw->rows, pw->cols, x, B, act_in, act_out, y, s),
                                     "gemv");
                        },
                        1, kOpGemv, 2.0 * B * static_cast<double>(pw->rows) * static_cast<double>(pw->cols), w.name});
}

void StepPlanner::add_gemm(const std::string& tag, const uint16_t* a, int64_t lda, int64_t K,
                                       const DevWeight* w0, const DevWeight* w1, std::vector<GemmGroup> groups,
                                       const EpilogueArgs& ep, int64_t N) {
  add_gemm_pieces(tag, a, lda, K, w0, w1, {groups}, ep, N, nullptr);
}

void StepPlanner::add_gemm_pieces(const std::string& tag, const uint16_t* a, int64_t lda, int64_t K,
                                              const DevWeight* w0, const DevWeight* w1,
                                              const std::vector<std::vector<GemmGroup>>& pieces, const EpilogueArgs& ep,
                                              int64_t N, const std::function<void(int)>& before_piece) {
  if (w0->cols != K || (w1 && (w1->cols != K || w1->rows != w0->rows)) || w0->rows != N)
    fail(DCPP_ERR_STATE, "internal: GEMM shape mismatch for " + w0->name);
  std::vector<GemmGroup> groups;
  for (auto& pg : pieces) groups.insert(groups.end(), pg.begin(), pg.end());
  // Fused dequantisation when every weight of the launch is packed and of
  // one quantised type; otherwise expand to bf16 first (or use bf16 as is).
  const AgWait ag = next_ag_;
  next_ag_ = AgWait{};
  const bool fused = w0->packed && (!w1 || (w1->packed && w1->type == w0->type));
  if (fused && ag.flags) fail(DCPP_ERR_STATE, "internal: arrival waits are not built for the fused-dequant GEMM");
  int64_t total_rows = 0;
  for (auto& g : groups) total_rows += g.rows;
  const bool pair = ctx_.use_pair(total_rows, fused);
  const int tile_m = pair ? 256 : kGemmBM;
  // N tile (bf16 B): 256 columns.  128-column tiles fill the waves of CTA
  // pairs better for some shapes (N = 2560 at M = 2048: 160 tiles for 74
  // pairs instead of 80) but measured slower there (each K block then feeds
  // half the MMA work per A tile loaded); DCPP_GEMM_TILE_N = 128 selects them.
  int tile_n = kGemmBN;
  if (!fused) {
    if (const char* f = getenv("DCPP_GEMM_TILE_N")) {
      const int v = atoi(f);
      if (v == 128 || v == kGemmBN) tile_n = v;
    }
  }
  if (fused) {
    int64_t a_rows = 0;
    for (auto& g : groups) a_rows = std::max<int64_t>(a_rows, g.row0 + g.rows);
    auto st = std::make_shared<CUtensorMap>();
    cuda_check(make_tmap_bf16(st.get(), a, K, a_rows, lda, kGemmBM), "tensor map A");
    const int bsrc = w0->type == kTypeQ4_K ? kBSrcQ4_K : kBSrcQ8_0;
    Ctx* c = &ctx_;
    for (size_t p = 0; p < pieces.size(); ++p) {
      if (before_piece) before_piece(static_cast<int>(p));
      const auto& pg = pieces[p];
      GemmArgs args{};
      args.N = static_cast<int32_t>(N);
      args.K = static_cast<int32_t>(K);
      if (pg.size() > static_cast<size_t>(kGemmMaxGroups)) fail(DCPP_ERR_UNSUPPORTED, "too many GEMM row groups");
      args.n_groups = static_cast<int32_t>(pg.size());
      for (size_t i = 0; i < pg.size(); ++i) args.groups[i] = pg[i];
      args.ep = ep;
      args.err = ctx_.d_err;
      args.qb[0].packed = w0->packed;
      args.qb[1].packed = w1 ? w1->packed : w0->packed;
      gemm_finalize_groups(args, tile_m);
      double flops = 0.0;
      for (auto& g : pg) flops += 2.0 * g.rows * static_cast<double>(N) * static_cast<double>(K);
      building_->push_back({[st, args, c, bsrc, pair](cudaStream_t s) {
                              if (pair)
                                cuda_check(launch_gemm_pair(*st, *st, *st, args, bsrc, c->num_sms, s), "fused gemm (pair)");
                              else
                                cuda_check(launch_gemm(*st, *st, *st, args, bsrc, c->num_sms, s), "fused gemm");
                            },
                            1, kOpGemm, flops, tag + " (fused dequant)"});
    }
    return;
  }
  if (!w0->data || (w1 && !w1->data)) fail(DCPP_ERR_STATE, "internal: mixed packed / raw weights in " + w0->name);
  // Weights expanded ahead (add_prefetch): read the expansion, after it is done.
  const auto pf0 = prefetched_.find(w0);
  const auto pf1 = w1 ? prefetched_.find(w1) : prefetched_.end();
  const bool ahead0 = pf0 != prefetched_.end(), ahead1 = pf1 != prefetched_.end();
  cudaEvent_t ahead_ready[2] = {ahead0 ? pf0->second.ready : nullptr, ahead1 ? pf1->second.ready : nullptr};
  const bool expand0 = w0->type != kTypeBF16 && !ahead0, expand1 = w1 && w1->type != kTypeBF16 && !ahead1;
  const int pair_idx = scratch_pair_;
  if (expand0 || expand1) scratch_pair_ = (scratch_pair_ + 1) % n_scratch_;
  uint16_t* const* sc = wscratch_[pair_idx];
  const uint16_t* b0 = ahead0 ? pf0->second.dst : expand0 ? sc[0] : reinterpret_cast<const uint16_t*>(w0->data);
  const uint16_t* b1 = b0;
  if (w1) b1 = ahead1 ? pf1->second.dst : expand1 ? sc[1] : reinterpret_cast<const uint16_t*>(w1->data);
  int64_t a_rows = 0;
  for (auto& g : groups) a_rows = std::max<int64_t>(a_rows, g.row0 + g.rows);
  auto st = std::make_shared<std::array<CUtensorMap, 3>>();
  cuda_check(make_tmap_bf16(&(*st)[0], a, K, a_rows, lda, kGemmBM), "tensor map A");
  cuda_check(make_tmap_bf16(&(*st)[1], b0, K, N, K, pair ? tile_n / 2 : tile_n), "tensor map B0");
  cuda_check(make_tmap_bf16(&(*st)[2], b1, K, N, K, pair ? tile_n / 2 : tile_n), "tensor map B1");
  Ctx* c = &ctx_;
  // Weight expansion on the side stream: it waits only for the last GEMM
  // that read this scratch pair (two expanding GEMMs back), so it overlaps
  // the GEMMs, attention and norms in between; the GEMM waits for it.
  if (expand0 || expand1) {
    add_wait(scratch_free_[pair_idx] ? scratch_free_[pair_idx] : plan_start_, 1);
    for (int k = 0; k < 2; ++k) {
      const DevWeight* w = k == 0 ? w0 : w1;
      if (!(k == 0 ? expand0 : expand1)) continue;
      uint16_t* dst = sc[k];
      Op o{[w, dst](cudaStream_t s) {
             cuda_check(launch_dequant_bf16(w->type, w->data, w->rows * w->cols, dst, s), "dequant");
           },
           1, kOpDequant, 0.0, "dequant " + tag};
      o.stream = 1;
      building_->push_back(o);
    }
  }
  cudaEvent_t ready = nullptr;
  if (expand0 || expand1) {
    ready = plan_event();
    add_record(ready, 1);
  }
  // K split: a single-piece residual GEMM (h += acc, no gate) whose tiles
  // fill the waves of CTA pairs poorly (N = 2560 at M = 2048: 80 tiles for 74
  // pairs) runs as S K-slices writing f32 partials, then one reduce adds
  // them to h in slice order.  DCPP_GEMM_KSPLIT = 0 turns it off.
  int splits = 1;
  int64_t split_rows = 0;
  if (pair && pieces.size() == 1 && ep.mode == kEpiResidGate && !ep.gate[0] && !ep.gate[1] && N % 4 == 0 &&
      ep.ld_out % 4 == 0) {
    const char* f = getenv("DCPP_GEMM_KSPLIT");
    if (!f || atoi(f) != 0) {
      int64_t m_tiles = 0;
      for (auto& g : groups) {
        m_tiles += (g.rows + tile_m - 1) / tile_m;
        split_rows = std::max<int64_t>(split_rows, g.orow0 + g.rows);
      }
      const int64_t tiles = m_tiles * ((N + tile_n - 1) / tile_n);
      splits = gemm_choose_k_splits(tiles, ctx_.num_sms, split_rows, N, K, 4, 16, /*reduce_adds=*/true, 0.05);
      const size_t need = static_cast<size_t>(splits) * split_rows * N * 4;
      // Ops built earlier hold the workspace pointer: it may be replaced by
      // a larger one only while no split launch refers to it.  Otherwise
      // this GEMM runs unsplit.
      if (splits > 1 && need > split_ws_bytes_ && split_launches_ == 0) {
        if (split_ws_) cuda_check(cudaFree(split_ws_), "free split workspace");
        split_ws_ = nullptr;
        split_ws_bytes_ = 0;
        const size_t bytes = std::max<size_t>(need, size_t(64) << 20);
        cuda_check(cudaMalloc(&split_ws_, bytes), "split workspace");
        split_ws_bytes_ = bytes;
      }
      if (splits > 1 && need > split_ws_bytes_) splits = 1;
    }
  }
  for (size_t p = 0; p < pieces.size(); ++p) {
    if (before_piece) before_piece(static_cast<int>(p));
    if (p == 0 && ready) add_wait(ready, 0);
    if (p == 0) {
      if (ahead_ready[0]) add_wait(ahead_ready[0], 0);
      if (ahead_ready[1] && ahead_ready[1] != ahead_ready[0]) add_wait(ahead_ready[1], 0);
    }
    const auto& pg = pieces[p];
    GemmArgs args{};
    args.N = static_cast<int32_t>(N);
    args.K = static_cast<int32_t>(K);
    if (pg.size() > static_cast<size_t>(kGemmMaxGroups)) fail(DCPP_ERR_UNSUPPORTED, "too many GEMM row groups");
    args.n_groups = static_cast<int32_t>(pg.size());
    for (size_t i = 0; i < pg.size(); ++i) args.groups[i] = pg[i];
    args.ep = ep;
    args.err = ctx_.d_err;
    gemm_finalize_groups(args, tile_m, tile_n);
    if (ag.flags) {
      if (!pair || splits > 1 || pieces.size() != 1)
        fail(DCPP_ERR_STATE, "internal: the overlapped all-gather needs one unsplit CTA-pair GEMM launch");
      args.ag_flags = ag.flags;
      args.ag_step = ag.step;
      args.ag_site = ag.site;
      args.ag_rank = ag.rank;
      args.ag_n = ag.n;
      args.ag_rows = ag.rows;
      args.ag_ld = ag.ld;
      args.ag_a = ag.a;
      for (int j = 0; j < 8; ++j) {
        args.ag_a_peer[j] = ag.a_peer[j];
        args.ag_flags_peer[j] = ag.flags_peer[j];
      }
      args.ag_count = ag.count;
      // M tile by M tile within bands of N tiles whose weight stays in L2
      // (64 MB, as the default tile order budgets): the rows arrive in row
      // order, and the first band's sweep overlaps their arrival.
      const double b_col = static_cast<double>(tile_n) * K * 2.0 * (w1 && w1 != w0 ? 2 : 1);
      args.raster = 1;
      args.band = std::max(1, std::min(args.n_tiles_n, static_cast<int>(64.0 * (1 << 20) / b_col)));
    }
    if (splits > 1) {
      args.ep = EpilogueArgs{};
      args.ep.mode = kEpiF32;
      args.ep.out_f32 = split_ws_;
      args.ep.ld_out = N;
      gemm_set_k_splits(args, splits, split_rows * N);
      ++split_launches_;
    }
    double flops = 0.0;
    for (auto& g : pg) flops += 2.0 * g.rows * static_cast<double>(N) * static_cast<double>(K);
    building_->push_back({[st, args, c, pair](cudaStream_t s) {
                            if (pair)
                              cuda_check(launch_gemm_pair((*st)[0], (*st)[1], (*st)[2], args, kBSrcBf16, c->num_sms, s),
                                         "gemm (pair)");
                            else
                              cuda_check(launch_gemm((*st)[0], (*st)[1], (*st)[2], args, kBSrcBf16, c->num_sms, s),
                                         "gemm");
                          },
                          1, kOpGemm, flops, tag});
    if (splits > 1) {
      const float* ws = split_ws_;
      float* out = ep.out_f32;
      const int64_t ld_out = ep.ld_out, rows = split_rows, n = N, stride = split_rows * N;
      const int sp = splits;
      building_->push_back({[=](cudaStream_t s) {
                              cuda_check(launch_split_reduce(ws, sp, stride, rows, n, n, out, ld_out, s, /*add=*/true), "split reduce");
                            },
                            1, kOpOther, 0.0, tag + " split reduce"});
    }
  }
  if (expand0 || expand1) {
    scratch_free_[pair_idx] = plan_event();
    add_record(scratch_free_[pair_idx], 0);
  }
}

void StepPlanner::run_ops(std::vector<Op>& ops, cudaGraphExec_t* graph) {
  cudaStream_t s = ctx_.stream;
  last_ops_ = &ops;
  auto issue = [&]() {
    if (!profiling_) {
      for (auto& o : ops) o.fn(op_stream(o.stream));
      return;
    }
    if (ev_.size() < 2 * ops.size()) {
      for (size_t i = ev_.size(); i < 2 * ops.size(); ++i) {
        cudaEvent_t e;
        cuda_check(cudaEventCreate(&e), "cudaEventCreate");
        ev_.push_back(e);
      }
    }
    // Inside a capture the records become graph event nodes (external
    // flag); outside they are ordinary stream records.
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cuda_check(cudaStreamIsCapturing(s, &cs), "cudaStreamIsCapturing");
    const unsigned flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
    for (size_t i = 0; i < ops.size(); ++i) {
      cudaStream_t os = op_stream(ops[i].stream);
      if (!ops[i].timed) {  // stream record / wait
        ops[i].fn(os);
        continue;
      }
      cuda_check(cudaEventRecordWithFlags(ev_[2 * i], os, flags), "event record");
      ops[i].fn(os);
      cuda_check(cudaEventRecordWithFlags(ev_[2 * i + 1], os, flags), "event record");
    }
  };
  if (!use_graph_) {
    issue();
    return;
  }
  if (!*graph) {
    cudaGraph_t g = nullptr;
    cuda_check(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal), "begin capture");
    try {
      issue();
    } catch (...) {
      cudaStreamEndCapture(s, &g);
      if (g) cudaGraphDestroy(g);
      throw;
    }
    cuda_check(cudaStreamEndCapture(s, &g), "end capture");
    cudaError_t e = cudaGraphInstantiate(graph, g, 0);
    cudaGraphDestroy(g);
    cuda_check(e, "graph instantiate");
  }
  cuda_check(cudaGraphLaunch(*graph, s), "graph launch");
}

void StepPlanner::profile(int kind, double* ms, double* flops, int64_t* launches) {
  if (!profiling_) fail(DCPP_ERR_STATE, "profiling is off (turn it on before prepare)");
  if (!last_ops_) fail(DCPP_ERR_STATE, "no step has run yet");
  cuda_check(cudaStreamSynchronize(ctx_.stream), "sync");
  double t = 0.0, f = 0.0;
  int64_t n = 0;
  for (size_t i = 0; i < last_ops_->size(); ++i) {
    const Op& o = (*last_ops_)[i];
    if (o.kind != kind || !o.timed) continue;
    float e = 0.f;
    cuda_check(cudaEventElapsedTime(&e, ev_[2 * i], ev_[2 * i + 1]), "cudaEventElapsedTime");
    t += e;
    f += o.flops;
    n += o.launches;
  }
  if (ms) *ms = t;
  if (flops) *flops = f;
  if (launches) *launches = n;
  // DCPP_PROFILE_OPS=<path>: also write every op of the step (index, tag,
  // kind, milliseconds, algorithmic FLOPs) as CSV, once per executed step.
  const char* path = getenv("DCPP_PROFILE_OPS");
  if (path && kind == kOpGemm) {
    FILE* f = fopen(path, "w");
    if (f) {
      fprintf(f, "index,tag,kind,ms,flops,stream\n");
      for (size_t i = 0; i < last_ops_->size(); ++i) {
        const Op& o = (*last_ops_)[i];
        if (!o.timed) continue;
        float e = 0.f;
        cudaEventElapsedTime(&e, ev_[2 * i], ev_[2 * i + 1]);
        fprintf(f, "%zu,%s,%d,%.5f,%.6g,%d\n", i, o.tag.c_str(), o.kind, e, o.flops, o.stream);
      }
      fclose(f);
    }
  }
}

}  // namespace dcpp
