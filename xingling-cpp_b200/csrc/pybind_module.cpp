// Python module `llm_cpp_engine`: the reference's pybind11 surface
// (src/bindings.cpp:7-39) over the C ABI of libxl_engine.so.
//
// Same class, method names, overload order (list before int), keyword names
// and defaults.  Differences: the device string is "cuda" or "cuda:N"
// ("cpu" raises ValueError: there is no CPU path in this engine); errors
// raise Python exceptions instead of exiting the process; the GIL is released
// while a token is computed.  Extensions: tensor-parallel construction,
// uniform / seed control, logits and KV read-back, device timing.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <string>
#include <vector>

#include "xl_engine.h"

namespace py = pybind11;

namespace {

[[noreturn]] void raise_status(int rc) {
    const std::string msg = xl_last_error();
    switch (rc) {
        case XL_ERR_ARG:
        case XL_ERR_TOKEN:
            throw py::value_error(msg);
        default:  // XL_ERR_IO too: the reference's Tensor::load throws std::runtime_error (src/tensor.cu:116,121)
            throw std::runtime_error(msg.empty() ? ("xl status " + std::to_string(rc)) : msg);
    }
}

void check(int rc) {
    if (rc != XL_OK) raise_status(rc);
}

int parse_device(const std::string& device) {
    if (device == "cuda") return 0;
    if (device.rfind("cuda:", 0) == 0) {
        try {
            size_t used = 0;
            const int d = std::stoi(device.substr(5), &used);
            if (used == device.size() - 5 && d >= 0) return d;
        } catch (const std::exception&) {
        }
    }
    if (device == "cpu")
        throw py::value_error("device 'cpu' is not supported: this engine runs on CUDA devices only (use 'cuda')");
    throw py::value_error("Invalid device: " + device);
}

class InferenceEngine {
   public:
    InferenceEngine(const std::string& device, int tp, int rank, py::bytes nccl_id, int layers, int vocab,
                    int max_ctx, int hidden, int heads, int ffn)
        : device_(device) {
        const int dev = parse_device(device);
        xl_config cfg;
        xl_config_default(&cfg);
        if (layers > 0) cfg.layers = layers;
        if (vocab > 0) cfg.vocab = vocab;
        if (max_ctx > 0) cfg.max_ctx = max_ctx;
        if (hidden > 0) cfg.hidden = hidden;
        if (heads > 0) cfg.heads = heads;
        if (ffn > 0) cfg.ffn = ffn;
        std::string id = nccl_id;
        if (tp > 1 && id.size() != XL_NCCL_ID_BYTES)
            throw py::value_error("nccl_id must hold the 128 bytes of llm_cpp_engine.nccl_unique_id()");
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_create(&cfg, dev, tp, rank, tp > 1 ? id.data() : nullptr, &e_);
        }
        check(rc);
    }
    ~InferenceEngine() { xl_engine_destroy(e_); }
    InferenceEngine(const InferenceEngine&) = delete;
    InferenceEngine& operator=(const InferenceEngine&) = delete;

    void load(const std::string& path) {
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_load(e_, path.c_str());
        }
        check(rc);
    }

    void to(const std::string& device) {
        if (parse_device(device) != parse_device(device_))
            throw py::value_error("moving an engine between devices is not supported; create one per device");
    }

    std::string device() const { return device_; }

    int next_token_prefill(const std::vector<int>& ids, float temperature, float top_p, float rp) {
        int tok = -1, rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_prefill(e_, ids.data(), static_cast<int>(ids.size()), temperature, top_p, rp, &tok);
        }
        check(rc);
        return tok;
    }

    int extend(const std::vector<int>& ids, float temperature, float top_p, float rp) {
        int tok = -1, rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_extend(e_, ids.data(), static_cast<int>(ids.size()), temperature, top_p, rp, &tok);
        }
        check(rc);
        return tok;
    }

    int next_token_decode(int token, float temperature, float top_p, float rp) {
        int tok = -1, rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_decode(e_, token, temperature, top_p, rp, &tok);
        }
        check(rc);
        return tok;
    }

    std::vector<int> generate(int token, int n, float temperature, float top_p, float rp, int stop_id) {
        if (n < 0) throw py::value_error("generate: n must be >= 0");
        std::vector<int> out(static_cast<size_t>(n));
        int got = 0, rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_generate(e_, token, n, temperature, top_p, rp, stop_id, out.data(), &got);
        }
        check(rc);
        out.resize(static_cast<size_t>(got));
        return out;
    }

    void set_uniforms(const std::vector<float>& u) { check(xl_engine_set_uniforms(e_, u.data(), static_cast<int>(u.size()))); }
    void seed(unsigned long long s) { check(xl_engine_seed(e_, s)); }

    py::tuple vocab_shard() const {
        int b = 0, c = 0;
        check(xl_engine_vocab_shard(e_, &b, &c));
        return py::make_tuple(b, c);
    }

    py::bytes last_logits() {
        int b = 0, c = 0;
        check(xl_engine_vocab_shard(e_, &b, &c));
        std::string buf(static_cast<size_t>(c) * sizeof(float), '\0');
        check(xl_engine_last_logits(e_, reinterpret_cast<float*>(&buf[0]), c));
        return py::bytes(buf);
    }

    py::tuple kv(int layer, int npos, int heads_local) {
        const size_t count = static_cast<size_t>(npos) * heads_local * 64;
        std::string k(count * sizeof(float), '\0'), v(count * sizeof(float), '\0');
        check(xl_engine_kv_copy(e_, layer, npos, reinterpret_cast<float*>(&k[0]), reinterpret_cast<float*>(&v[0])));
        return py::make_tuple(py::bytes(k), py::bytes(v));
    }

    int ctx_len() const { return xl_engine_ctx_len(e_); }

    float last_device_ms() const {
        float ms = 0.0f;
        check(xl_engine_last_device_ms(e_, &ms));
        return ms;
    }

    float last_kernel_ms() const {
        float ms = 0.0f;
        check(xl_engine_last_kernel_ms(e_, &ms));
        return ms;
    }

    float last_load_s() const {
        float sec = 0.0f;
        check(xl_engine_last_load_s(e_, &sec));
        return sec;
    }

    void set_option(const std::string& key, int value) {
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_set_option(e_, key.c_str(), value);
        }
        check(rc);
    }

    py::bytes phase_trace(int n) {
        std::string buf(static_cast<size_t>(n) * 8, '\0');
        check(xl_engine_phase_trace(e_, reinterpret_cast<unsigned long long*>(&buf[0]), n));
        return py::bytes(buf);
    }

    float profile_lm_head(int iters) {
        float ms = 0.0f;
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_engine_profile_lm_head(e_, iters, &ms);
        }
        check(rc);
        return ms;
    }

    // Special ids of src/inference.cu:32-36 (plain attributes, unused by the engine).
    int im_start_id = 151644;
    int im_end_id = 151645;
    int nl_id = 198;
    int role_id_user = 872;
    int role_id_assistant = 77091;

    xl_engine* handle() const { return e_; }

   private:
    xl_engine* e_ = nullptr;
    std::string device_;
};

// XL_BATCH sequences decoding together over an InferenceEngine's weights (no
// reference counterpart; see xl_batch_* in xl_engine.h).
class BatchDecoder {
   public:
    explicit BatchDecoder(InferenceEngine& eng) {
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_batch_create(eng.handle(), &b_);
        }
        check(rc);
    }
    ~BatchDecoder() { xl_batch_destroy(b_); }
    BatchDecoder(const BatchDecoder&) = delete;
    BatchDecoder& operator=(const BatchDecoder&) = delete;

    void seed(int seq, unsigned long long s) { check(xl_batch_seed(b_, seq, s)); }

    int prefill(int seq, const std::vector<int>& ids, float temperature, float top_p, float repetition_penalty) {
        int tok = 0, rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_batch_prefill(b_, seq, ids.data(), static_cast<int>(ids.size()), temperature, top_p,
                                  repetition_penalty, &tok);
        }
        check(rc);
        return tok;
    }

    std::vector<int> step(const std::vector<int>& tokens, float temperature, float top_p, float repetition_penalty) {
        if (tokens.size() != XL_BATCH) throw py::value_error("step: one token per sequence (" +
                                                             std::to_string(XL_BATCH) + ")");
        std::vector<int> out(XL_BATCH);
        int rc;
        {
            py::gil_scoped_release nogil;
            rc = xl_batch_decode(b_, tokens.data(), temperature, top_p, repetition_penalty, out.data());
        }
        check(rc);
        return out;
    }

    py::bytes last_logits(int seq, int vocab) {
        std::string buf(static_cast<size_t>(vocab) * sizeof(float), '\0');
        check(xl_batch_last_logits(b_, seq, reinterpret_cast<float*>(&buf[0]), vocab));
        return py::bytes(buf);
    }

    int ctx_len(int seq) const { return xl_batch_ctx_len(b_, seq); }

    float last_device_ms() const {
        float ms = 0.0f;
        check(xl_batch_last_device_ms(b_, &ms));
        return ms;
    }

   private:
    xl_batch* b_ = nullptr;
};

}  // namespace

PYBIND11_MODULE(llm_cpp_engine, m) {
    m.doc() = "XingLing-0.68B token loop on NVIDIA B200 (sm_100a), drop-in for the reference's llm_cpp_engine";

    py::class_<BatchDecoder>(m, "BatchDecoder")
        .def(py::init<InferenceEngine&>(), py::arg("engine"), py::keep_alive<1, 2>())
        .def_property_readonly_static("size", [](py::object) { return XL_BATCH; })
        .def("seed", &BatchDecoder::seed, py::arg("seq"), py::arg("seed"))
        .def("prefill", &BatchDecoder::prefill, py::arg("seq"), py::arg("input_ids"), py::arg("temperature") = 0.7f,
             py::arg("top_p") = 0.9f, py::arg("repetition_penalty") = 1.1f)
        .def("step", &BatchDecoder::step, py::arg("tokens"), py::arg("temperature") = 0.7f, py::arg("top_p") = 0.9f,
             py::arg("repetition_penalty") = 1.1f)
        .def("last_logits", &BatchDecoder::last_logits, py::arg("seq"), py::arg("vocab"))
        .def("ctx_len", &BatchDecoder::ctx_len, py::arg("seq"))
        .def("last_device_ms", &BatchDecoder::last_device_ms);

    m.def("kernel_launches", []() { return xl_kernel_launches(); },
          "Kernels this library has run in this process (decode-graph kernels count at each replay).");
    m.def("nccl_unique_id", []() {
        std::string id(XL_NCCL_ID_BYTES, '\0');
        check(xl_nccl_unique_id(&id[0], XL_NCCL_ID_BYTES));
        return py::bytes(id);
    });

    py::class_<InferenceEngine>(m, "InferenceEngine")
        .def(py::init<const std::string&, int, int, py::bytes, int, int, int, int, int, int>(),
             py::arg("device") = "cuda", py::arg("tp") = 1, py::arg("rank") = 0, py::arg("nccl_id") = py::bytes(),
             py::arg("layers") = 0, py::arg("vocab") = 0, py::arg("max_ctx") = 0, py::arg("hidden") = 0,
             py::arg("heads") = 0, py::arg("ffn") = 0)
        .def("load", &InferenceEngine::load, "load the raw-fp32 weight tree from a directory")
        .def("to", &InferenceEngine::to, "device check ('cuda' / 'cuda:N'); engines do not move")
        .def("device", &InferenceEngine::device, "the engine's device string")
        .def("next_token", &InferenceEngine::next_token_prefill, py::arg("input_ids"), py::arg("temperature") = 0.7f,
             py::arg("top_p") = 0.9f, py::arg("repetition_penalty") = 1.1f)
        .def("next_token", &InferenceEngine::next_token_decode, py::arg("token"), py::arg("temperature") = 0.7f,
             py::arg("top_p") = 0.9f, py::arg("repetition_penalty") = 1.1f)
        .def("extend", &InferenceEngine::extend, py::arg("input_ids"), py::arg("temperature") = 0.7f,
             py::arg("top_p") = 0.9f, py::arg("repetition_penalty") = 1.1f,
             "prefill continuation: the ids extend the cached sequence (the repetition set is kept)")
        .def("generate", &InferenceEngine::generate, py::arg("token"), py::arg("n"), py::arg("temperature") = 0.7f,
             py::arg("top_p") = 0.9f, py::arg("repetition_penalty") = 1.1f, py::arg("stop_id") = -1,
             "up to n decode steps fed on the device; stops after stop_id (returned) or a full cache")
        .def("set_uniforms", &InferenceEngine::set_uniforms, py::arg("uniforms"))
        .def("seed", &InferenceEngine::seed, py::arg("seed"))
        .def("vocab_shard", &InferenceEngine::vocab_shard)
        .def("last_logits", &InferenceEngine::last_logits)
        .def("kv", &InferenceEngine::kv, py::arg("layer"), py::arg("npos"), py::arg("heads_local"))
        .def("ctx_len", &InferenceEngine::ctx_len)
        .def("last_device_ms", &InferenceEngine::last_device_ms)
        .def("last_kernel_ms", &InferenceEngine::last_kernel_ms)
        .def("last_load_s", &InferenceEngine::last_load_s)
        .def("set_option", &InferenceEngine::set_option, py::arg("key"), py::arg("value"))
        .def("phase_trace", &InferenceEngine::phase_trace, py::arg("n"))
        .def("profile_lm_head", &InferenceEngine::profile_lm_head, py::arg("iters") = 20)
        .def_readwrite("im_start_id", &InferenceEngine::im_start_id)
        .def_readwrite("im_end_id", &InferenceEngine::im_end_id)
        .def_readwrite("nl_id", &InferenceEngine::nl_id)
        .def_readwrite("role_id_user", &InferenceEngine::role_id_user)
        .def_readwrite("role_id_assistant", &InferenceEngine::role_id_assistant);
}
