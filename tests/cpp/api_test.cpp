// Exercises the C++ surface (include/dcpp.hpp) the way a diffusers-cpp
// caller would.  Built and run by tests/test_cpp_api.py.
//   api_test cpu <config.json>                      host-only checks (no GPU)
//   api_test gpu <params.bin> <inputs.bin> <out.bin> one denoise step on GPU 0
#include <cstdio>
#include <cstring>
#include <fstream>
#include <iostream>
#include <string>
#include <vector>

#include "dcpp.hpp"

static int fails = 0;
#define EXPECT(c)                                                      \
    do {                                                               \
        if (!(c)) {                                                    \
            std::cerr << "FAILED " << __LINE__ << ": " #c << std::endl; \
            ++fails;                                                   \
        }                                                              \
    } while (0)

struct Reader {
    std::ifstream f;
    explicit Reader(const char* p) : f(p, std::ios::binary) {}
    template <class T>
    T get() {
        T v{};
        f.read(reinterpret_cast<char*>(&v), sizeof(T));
        return v;
    }
    std::vector<char> bytes(size_t n) {
        std::vector<char> b(n);
        f.read(b.data(), static_cast<std::streamsize>(n));
        return b;
    }
};

static int cpu_mode(const char* config_path) {
    auto cfg = dcpp::Flux2Transformer2DModel::Config::from_file(config_path);
    EXPECT(cfg.num_layers == 1 && cfg.num_single_layers == 1 && cfg.num_attention_heads == 6);
    EXPECT(cfg.attention_head_dim == 128 && cfg.rope_theta == 2000);  // defaults kept

    EXPECT((dcpp::ShardingPlan::split(24, 5) == std::vector<int64_t>{4, 5, 5, 5, 5}));
    EXPECT((dcpp::ShardingPlan::split(6, 2, {2.f, 1.f}) == std::vector<int64_t>{4, 2}));

    dcpp::FlowMatchEulerDiscreteScheduler sch;
    auto sched = sch.pipeline_schedule(4, 4096);  // default: static shift 1, mu unused
    EXPECT(sched.first.size() == 4 && sched.second.size() == 5);
    EXPECT(sched.first[0] == 1000.f && sched.second[2] == 0.5f && sched.second[4] == 0.f);
    auto lin = sch.schedule(2);  // sigma_max .. sigma_min
    EXPECT(lin.second[0] == 1.f && lin.second[1] == 0.001f && lin.second[2] == 0.f);
    sch.use_dynamic_shifting = true;
    sch.time_shift_type = "linear";
    auto dyn = sch.schedule(2, 1.0f, {0.5f, 0.25f});  // mu = 1, linear: the identity
    EXPECT(dyn.second[0] == 0.5f && dyn.second[1] == 0.25f);
    sch.time_shift_type = "cubic";
    {
        bool bad = false;
        try {
            sch.schedule(2);
        } catch (const dcpp::Error& e) {
            bad = e.status == DCPP_ERR_INVALID_ARG;
        }
        EXPECT(bad);
    }
    EXPECT(dcpp::compute_empirical_mu(8192, 4) == 0.00016927f * 8192.f + 0.45666666f);
    auto img = dcpp::prepare_img_ids(1, 2, 3);
    EXPECT(img.size() == 24 && img[4 * 5 + 1] == 1 && img[4 * 5 + 2] == 2 && img[4 * 5 + 0] == 0);
    auto txt = dcpp::prepare_txt_ids(2, 3);
    EXPECT(txt.size() == 24 && txt[4 * 5 + 3] == 2);
    auto refi = dcpp::prepare_ref_image_ids(1, {{1, 2}, {2, 1}});
    EXPECT(refi.size() == 16 && refi[0] == 10 && refi[4 * 3 + 0] == 20 && refi[4 * 3 + 1] == 1);

    dcpp::Flux2Transformer2DModel host(nullptr, cfg);  // loader / shard layout only
    host.set_sharding(1, 2, {2.f, 1.f});
    auto s = host.shard();
    EXPECT((s == std::vector<int64_t>{4, 2, 1536, 768}));
    std::string first;
    EXPECT(host.missing(&first) > 0 && !first.empty());
    bool threw = false;
    try {
        host.prepare(1, 16, 8);
    } catch (const dcpp::Error& e) {
        threw = e.status == DCPP_ERR_STATE;
    }
    EXPECT(threw);
    try {
        dcpp::Flux2Transformer2DModel::Config::from_file("/nonexistent/config.json");
        EXPECT(false);
    } catch (const dcpp::Error& e) {
        EXPECT(e.status == DCPP_ERR_NOT_FOUND);
    }
    return fails;
}

static int gpu_mode(const char* params_path, const char* inputs_path, const char* out_path) {
    Reader in(inputs_path);
    const int64_t n_layers = in.get<int64_t>(), n_single = in.get<int64_t>(), heads = in.get<int64_t>();
    const int64_t jd = in.get<int64_t>(), in_ch = in.get<int64_t>();
    const int64_t n_img = in.get<int64_t>(), n_ref = in.get<int64_t>(), n_txt = in.get<int64_t>();
    const float sigma = in.get<float>(), dt = in.get<float>();
    auto lat = in.bytes(n_img * in_ch * 4), ref = in.bytes(n_ref * in_ch * 4), enc = in.bytes(n_txt * jd * 4);
    auto img_ids = in.bytes(n_img * 16), ref_ids = in.bytes(n_ref * 16), txt_ids = in.bytes(n_txt * 16);

    dcpp::Flux2Transformer2DModel::Config cfg;
    cfg.num_layers = n_layers;
    cfg.num_single_layers = n_single;
    cfg.num_attention_heads = heads;
    cfg.joint_attention_dim = jd;
    cfg.in_channels = in_ch;
    cfg.guidance_embeds = 0;
    dcpp::CudaRuntime rt(0);
    dcpp::Flux2Transformer2DModel dit(&rt, cfg);
    Reader pr(params_path);
    const int64_t n_params = pr.get<int64_t>();
    for (int64_t i = 0; i < n_params; ++i) {
        auto name = pr.bytes(pr.get<int64_t>());
        const int type = static_cast<int>(pr.get<int64_t>());
        std::vector<int64_t> shape(static_cast<size_t>(pr.get<int64_t>()));
        for (auto& d : shape) d = pr.get<int64_t>();
        auto data = pr.bytes(pr.get<int64_t>());
        dit.set_param(std::string(name.begin(), name.end()), type, shape, data.data(), data.size());
    }
    EXPECT(dit.missing() == 0);
    dit.prepare(1, n_img, n_txt, n_ref);
    dcpp::Flux2KleinPipeline pipe{dit};
    std::vector<float> out(static_cast<size_t>(n_img * in_ch));
    pipe.denoise(reinterpret_cast<const float*>(lat.data()), reinterpret_cast<const float*>(enc.data()),
                 reinterpret_cast<const int32_t*>(img_ids.data()), reinterpret_cast<const int32_t*>(txt_ids.data()),
                 n_ref ? reinterpret_cast<const float*>(ref.data()) : nullptr,
                 n_ref ? reinterpret_cast<const int32_t*>(ref_ids.data()) : nullptr, &sigma, dt, out.data());
    std::ofstream o(out_path, std::ios::binary);
    o.write(reinterpret_cast<const char*>(out.data()), static_cast<std::streamsize>(out.size() * 4));
    return fails;
}

int main(int argc, char** argv) {
    try {
        if (argc >= 3 && std::string(argv[1]) == "cpu") return cpu_mode(argv[2]) ? 1 : 0;
        if (argc >= 5 && std::string(argv[1]) == "gpu") return gpu_mode(argv[2], argv[3], argv[4]) ? 1 : 0;
    } catch (const dcpp::Error& e) {
        std::cerr << "dcpp::Error " << e.status << ": " << e.what() << std::endl;
        return 2;
    }
    std::cerr << "usage: api_test cpu <config.json> | gpu <params.bin> <inputs.bin> <out.bin>" << std::endl;
    return 3;
}
