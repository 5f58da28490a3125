/*
 * dcpp.hpp -- C++ module / pipeline surface over the C ABI (dcpp.h).
 *
 * Header-only.  It gives a C++ caller of diffusers-cpp the shapes it already
 * uses, backed by the B200 kernels:
 *   dcpp::CudaRuntime                       the op backend: a GPU context whose
 *                                           methods are the Runtime ops this
 *                                           library executes (src/ggml/Runtime.hpp:
 *                                           mul_mat :136, norm :250, rms_norm :273,
 *                                           rope_ext :277, flash_attn_ext :281),
 *                                           eagerly on device buffers
 *   dcpp::ShardingPlan                      the sharding planner's tensor_split
 *                                           rounding (ShardingRuntime.cpp:280-296)
 *   dcpp::Flux2Transformer2DModel           Flux2Transformer2DModel (Config,
 *                                           from_file, from_pretrained, forward;
 *                                           Flux2Transformer2DModel.hpp:10-50)
 *   dcpp::FlowMatchEulerDiscreteScheduler   schedule with every constructor option
 *                                           (FlowMatchEulerDiscreteScheduler.cpp:8-208),
 *                                           and compute_empirical_mu
 *   dcpp::Flux2KleinPipeline                denoise (Flux2KleinPipeline.cpp:496-537),
 *                                           with or without reference images
 * Errors become dcpp::Error (a std::runtime_error carrying the status), as the
 * reference throws std::runtime_error.
 */
#ifndef DCPP_HPP
#define DCPP_HPP

#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "dcpp.h"

namespace dcpp {

struct Error : std::runtime_error {
    dcpp_status status;
    Error(dcpp_status s, const std::string& msg) : std::runtime_error(msg), status(s) {}
};

inline void check(dcpp_status s, const char* what, const char* detail = nullptr) {
    if (s != DCPP_OK)
        throw Error(s, std::string(what) + ": " + (detail ? detail : "status " + std::to_string(static_cast<int>(s))));
}

/* One GPU, one stream: the Backend / Device pair of the reference
 * (src/ggml/Backend.hpp:5-31) plus the ops it runs.  Pointers are device
 * pointers unless a method says otherwise. */
class CudaRuntime {
public:
    explicit CudaRuntime(int device = 0) {
        dcpp_status s = dcpp_init(device, &ctx_);
        if (s != DCPP_OK) {
            ctx_ = nullptr;
            check(s, "dcpp_init", "no usable B200 (sm_100a) device");
        }
    }
    ~CudaRuntime() {
        if (ctx_) dcpp_destroy(ctx_);
    }
    CudaRuntime(const CudaRuntime&) = delete;
    CudaRuntime& operator=(const CudaRuntime&) = delete;

    dcpp_ctx* handle() const { return ctx_; }
    void ok(dcpp_status s, const char* what) const { check(s, what, dcpp_last_error(ctx_)); }

    void set_stream(void* cuda_stream) { ok(dcpp_set_stream(ctx_, cuda_stream), "set_stream"); }
    void synchronize() { ok(dcpp_synchronize(ctx_), "synchronize"); }
    void* alloc(size_t bytes) {
        void* p = nullptr;
        ok(dcpp_alloc(ctx_, bytes, &p), "alloc");
        return p;
    }
    void free(void* p) { ok(dcpp_free(ctx_, p), "free"); }
    /* Host or device pointers on either side (UVA). */
    void memcpy(void* dst, const void* src, size_t bytes) { ok(dcpp_memcpy(ctx_, dst, src, bytes), "memcpy"); }

    /* Runtime::mul_mat(W, x) (Runtime.hpp:136, Linear::forward): y[M, N] f32 =
     * x[M, K] bf16 . W[N, K]^T, W of ggml type `wtype` (Q8_0, Q4_K, BF16, F16, F32). */
    void mul_mat(int wtype, const void* w, int64_t N, int64_t K, const uint16_t* x, int64_t M, float* y) {
        ok(dcpp_gemm(ctx_, wtype, w, N, K, x, M, y), "mul_mat");
    }
    /* Runtime::norm (Runtime.hpp:250) without affine, then the adaLN
     * modulation (1 + scale) x + shift: y bf16. */
    void norm_modulate(const float* x, int64_t rows, int64_t D, const float* shift, const float* scale, float eps,
                       uint16_t* y) {
        ok(dcpp_layernorm_mod(ctx_, x, rows, D, shift, scale, eps, y), "norm");
    }
    /* rms_norm (q, k) + rope_ext (NORMAL mode, per axis section) +
     * flash_attn_ext (Runtime.hpp:273, :277, :281), fused: see dcpp_attention. */
    void flash_attn_ext(const uint16_t* qkv, int64_t B, int64_t S, int64_t H, const float* norm_q,
                        const float* norm_k, float eps, const int32_t* ids, const std::vector<int64_t>& axes_dims,
                        float theta, uint16_t* out) {
        ok(dcpp_attention(ctx_, qkv, B, S, H, 128, norm_q, norm_k, eps, ids, static_cast<int>(axes_dims.size()),
                          axes_dims.data(), theta, out),
           "flash_attn_ext");
    }
    /* The meta backend's AllReduce at a P -> R bridge (ShardingRuntime.hpp:1082-1091). */
    void all_reduce(void* buf, int64_t count, int dtype) { ok(dcpp_allreduce(ctx_, buf, count, dtype), "all_reduce"); }
    /* Join the tensor-parallel group (one process per GPU); rank 0 makes the id. */
    static std::vector<char> unique_id() {
        std::vector<char> id(DCPP_NCCL_ID_BYTES);
        check(dcpp_tp_get_unique_id(id.data()), "tp_get_unique_id");
        return id;
    }
    void init_tensor_parallel(int rank, int nranks, const std::vector<char>& id) {
        ok(dcpp_tp_init(ctx_, rank, nranks, id.data()), "tp_init");
    }
    void set_wait_timeout(double seconds) { ok(dcpp_set_wait_timeout(ctx_, seconds), "set_wait_timeout"); }

private:
    dcpp_ctx* ctx_ = nullptr;
};

/* The sharding planner's split of `units` over the ranks in proportion to
 * tensor_split ratios (empty: equal). */
struct ShardingPlan {
    static std::vector<int64_t> split(int64_t units, int nranks, const std::vector<float>& ratios = {}) {
        std::vector<int64_t> out(static_cast<size_t>(nranks > 0 ? nranks : 0));
        check(dcpp_tp_plan_split(units, nranks, ratios.empty() ? nullptr : ratios.data(), out.data()), "plan_split");
        return out;
    }
};

class Flux2Transformer2DModel {
public:
    /* Flux2Transformer2DModel::Config: the same fields and defaults. */
    struct Config : dcpp_flux2_config {
        Config() { dcpp_flux2_config_default(this); }
        static Config from_file(const std::string& path) {
            Config c;
            check(dcpp_flux2_config_from_file(path.c_str(), &c), "Config::from_file", path.c_str());
            return c;
        }
    };

    /* A model on `rt` (device), or host-only when rt is null: the loader and
     * the shard layout without execution (dcpp_flux2_create_host). */
    Flux2Transformer2DModel(CudaRuntime* rt, const Config& cfg) : rt_(rt) {
        if (rt)
            rt->ok(dcpp_flux2_create(rt->handle(), &cfg, &m_), "Flux2Transformer2DModel");
        else
            check(dcpp_flux2_create_host(&cfg, &m_), "Flux2Transformer2DModel (host)");
    }
    /* Flux2KleinPipeline::from_pretrained's transformer folder: config.json + GGUF. */
    static Flux2Transformer2DModel from_pretrained(CudaRuntime& rt, const std::string& dir) {
        Flux2Transformer2DModel m;
        m.rt_ = &rt;
        rt.ok(dcpp_flux2_from_pretrained(rt.handle(), dir.c_str(), &m.m_), "from_pretrained");
        return m;
    }
    ~Flux2Transformer2DModel() {
        if (m_) dcpp_flux2_destroy(m_);
    }
    Flux2Transformer2DModel(Flux2Transformer2DModel&& o) noexcept : rt_(o.rt_), m_(o.m_) { o.m_ = nullptr; }
    Flux2Transformer2DModel(const Flux2Transformer2DModel&) = delete;
    Flux2Transformer2DModel& operator=(const Flux2Transformer2DModel&) = delete;

    dcpp_flux2* handle() const { return m_; }
    void ok(dcpp_status s, const char* what) const { check(s, what, dcpp_flux2_last_error(m_)); }

    /* Tensor parallelism per the planner (before parameters are set). */
    void set_sharding(int rank, int nranks, const std::vector<float>& tensor_split = {}) {
        ok(dcpp_flux2_set_tensor_split(m_, rank, nranks, tensor_split.empty() ? nullptr : tensor_split.data()),
           "set_sharding");
    }
    /* (first head, heads, first MLP feature, MLP features) of this rank. */
    std::vector<int64_t> shard() const {
        std::vector<int64_t> s(4);
        ok(dcpp_flux2_shard(m_, &s[0], &s[1], &s[2], &s[3]), "shard");
        return s;
    }
    /* Parameter::set by GGUF name (raw GGUF bytes, shape in PyTorch order). */
    void set_param(const std::string& name, int type, const std::vector<int64_t>& shape, const void* data,
                   size_t nbytes) {
        ok(dcpp_flux2_set_param(m_, name.c_str(), type, static_cast<int>(shape.size()), shape.data(), data, nbytes),
           "set_param");
    }
    int missing(std::string* first = nullptr) const {
        int n = 0;
        char buf[512] = {0};
        ok(dcpp_flux2_missing(m_, &n, buf, sizeof(buf)), "missing");
        if (first) *first = buf;
        return n;
    }
    void prepare(int64_t batch, int64_t n_img, int64_t n_txt, int64_t n_ref = 0, bool graph = true) {
        ok(dcpp_flux2_prepare_ref(m_, batch, n_img, n_ref, n_txt, graph ? 1 : 0), "prepare");
    }
    /* Flux2Transformer2DModel::forward (host or device pointers). */
    void forward(const float* hidden, const float* encoder, const float* timestep, const int32_t* img_ids,
                 const int32_t* txt_ids, const float* guidance, float* out) {
        ok(dcpp_flux2_forward(m_, hidden, encoder, timestep, img_ids, txt_ids, guidance, out), "forward");
    }

private:
    Flux2Transformer2DModel() = default;
    CudaRuntime* rt_ = nullptr;
    dcpp_flux2* m_ = nullptr;
};

/* The pipeline's RoPE position ids, int32 (t, h, w, l) per token,
 * batch-major (Flux2KleinPipeline.cpp:26-127). */
inline std::vector<int32_t> prepare_txt_ids(int64_t batch, int64_t seq_len) {
    std::vector<int32_t> ids(static_cast<size_t>(batch > 0 && seq_len > 0 ? batch * seq_len * 4 : 0));
    check(dcpp_flux2_prepare_txt_ids(batch, seq_len, ids.data()), "prepare_txt_ids");
    return ids;
}
inline std::vector<int32_t> prepare_img_ids(int64_t batch, int64_t packed_h, int64_t packed_w) {
    std::vector<int32_t> ids(
        static_cast<size_t>(batch > 0 && packed_h > 0 && packed_w > 0 ? batch * packed_h * packed_w * 4 : 0));
    check(dcpp_flux2_prepare_img_ids(batch, packed_h, packed_w, ids.data()), "prepare_img_ids");
    return ids;
}
/* packed_sizes: (h, w) of each reference image (its size / (VAE scale factor * 2)). */
inline std::vector<int32_t> prepare_ref_image_ids(int64_t batch, const std::vector<std::pair<int64_t, int64_t>>& packed_sizes) {
    std::vector<int64_t> hw;
    int64_t tokens = 0;
    for (const auto& s : packed_sizes) {
        hw.push_back(s.first);
        hw.push_back(s.second);
        tokens += s.first * s.second;
    }
    std::vector<int32_t> ids(static_cast<size_t>(batch > 0 && tokens > 0 ? batch * tokens * 4 : 0));
    check(dcpp_flux2_prepare_ref_image_ids(batch, static_cast<int64_t>(packed_sizes.size()), hw.data(), ids.data()),
          "prepare_ref_image_ids");
    return ids;
}

/* The pipeline's compute_empirical_mu (Flux2KleinPipeline.cpp:130-141). */
inline float compute_empirical_mu(int64_t image_seq_len, int num_steps) {
    float mu = 0.f;
    check(dcpp_flux2_empirical_mu(image_seq_len, num_steps, &mu), "compute_empirical_mu");
    return mu;
}

/* FlowMatchEulerDiscreteScheduler: the constructor's options with the
 * reference's defaults (FlowMatchEulerDiscreteScheduler.hpp:11-18). */
struct FlowMatchEulerDiscreteScheduler {
    int num_train_timesteps = 1000;
    float shift = 1.0f;
    bool use_dynamic_shifting = false;
    bool has_shift_terminal = false;
    float shift_terminal = 0.0f;
    bool invert_sigmas = false;
    std::string time_shift_type = "exponential";

    /* schedule(num_inference_steps, mu, sigmas) (FlowMatchEulerDiscreteScheduler.hpp:20-24):
     * n timesteps and n + 1 sigmas; empty sigmas: n points from sigma_max
     * down to sigma_min. */
    std::pair<std::vector<float>, std::vector<float>> schedule(int n, float mu = 0.0f,
                                                               const std::vector<float>& sigmas = {}) const {
        dcpp_flow_match_config c;
        dcpp_flow_match_config_default(&c);
        c.num_train_timesteps = num_train_timesteps;
        c.shift = shift;
        c.use_dynamic_shifting = use_dynamic_shifting ? 1 : 0;
        c.has_shift_terminal = has_shift_terminal ? 1 : 0;
        c.shift_terminal = shift_terminal;
        c.invert_sigmas = invert_sigmas ? 1 : 0;
        if (time_shift_type == "linear")
            c.time_shift_type = DCPP_TIME_SHIFT_LINEAR;
        else if (time_shift_type != "exponential")
            throw Error(DCPP_ERR_INVALID_ARG, "unsupported time_shift_type: " + time_shift_type);
        if (!sigmas.empty() && sigmas.size() != static_cast<size_t>(n))
            throw Error(DCPP_ERR_INVALID_ARG, "schedule: sigmas must have num_inference_steps entries");
        std::vector<float> t(static_cast<size_t>(n > 0 ? n : 0)), s(static_cast<size_t>(n > 0 ? n + 1 : 0));
        check(dcpp_flow_match_schedule_ex(&c, n, mu, sigmas.empty() ? nullptr : sigmas.data(), t.data(), s.data()),
              "schedule");
        return {t, s};
    }
    /* The pipeline's denoise schedule (Flux2KleinPipeline.cpp:348-358):
     * sigmas 1 - i/n and mu = compute_empirical_mu(image_seq_len, n). */
    std::pair<std::vector<float>, std::vector<float>> pipeline_schedule(int n, int64_t image_seq_len) const {
        std::vector<float> base(static_cast<size_t>(n > 0 ? n : 0));
        for (int i = 0; i < n; ++i) base[static_cast<size_t>(i)] = static_cast<float>(1.0 - static_cast<double>(i) / n);
        return schedule(n, compute_empirical_mu(image_seq_len, n), base);
    }
};

/* Flux2KleinPipeline::denoise for one step of a prepared transformer.
 * image_latents / image_latent_ids: the reference images (both null for
 * text-to-image).  timestep is sigma (the pipeline's timestep / 1000). */
struct Flux2KleinPipeline {
    Flux2Transformer2DModel& transformer;
    void denoise(const float* latents, const float* prompt_embeds, const int32_t* img_ids, const int32_t* txt_ids,
                 const float* image_latents, const int32_t* image_latent_ids, const float* timestep, float dt,
                 float* latents_out) {
        transformer.ok(dcpp_flux2_denoise_step_ref(transformer.handle(), latents, image_latents, image_latent_ids,
                                                   prompt_embeds, timestep, dt, img_ids, txt_ids, latents_out),
                       "denoise");
    }
};

}  // namespace dcpp

#endif /* DCPP_HPP */
