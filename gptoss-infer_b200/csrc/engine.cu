// Decode engine (see engine.h): checkpoint loading, the per-token step as one CUDA graph, scoring.
//
// Per step (token in device memory, position in device memory, so one captured graph serves every step):
//   x = embed[token]
//   per layer: qkv = Wqkv RMSNorm(x; ln1) + bqkv            (GEMV with the norm fused in front)
//              attn = attention(RoPE(q), cache + RoPE(k), v)   (one launch: RoPE, fp16 cache append, split-K
//                                                              partials, merge with the sinks by the last CTA)
//              x += Wo attn + bo                               (GEMV with the residual fused)
//              x += MoE(RMSNorm(x; ln2))                       (the fused tensor-core decode MoE kernel)
//   logits = lm_head RMSNorm(x; norm); position += 1
// This is the layer sequence of openvang/gptoss-infer runtime/src/engine.cu:242-262 (and of the fp32 reference
// gptoss_ref/model.py:107-125), with RMSNorms fused into their consumers and the MoE in one kernel. With
// gptoss_set_attention_impl(1) the first three lines of a layer run as one cooperative launch (attn_block.cu).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <filesystem>
#include <fstream>
#include <map>
#include <sstream>
#include <stdexcept>

#include "common.cuh"
#include "engine.h"
#include "json_min.h"
#include "kernels.h"

namespace gpt {

namespace {

std::string read_text(const std::string& path) {
    std::ifstream f(path);
    if (!f) throw std::runtime_error("cannot read " + path);
    std::stringstream ss;
    ss << f.rdbuf();
    return ss.str();
}

bool file_exists(const std::string& path) {
    struct stat st;
    return ::stat(path.c_str(), &st) == 0;
}

// ---------------------------------------------------------------------------------------------------- safetensors
// A checkpoint directory: model.safetensors.index.json (weight_map: tensor -> file), else every *.safetensors file
// in it. Each file is an 8-byte little-endian header length, a JSON header (name -> dtype, shape, data_offsets
// relative to the data start) and the data; the files are memory-mapped read-only while the engine loads.
struct TensorRef {
    const uint8_t* data = nullptr;
    size_t nbytes = 0;
    std::string dtype;
    std::vector<long long> shape;
};

class Checkpoint {
  public:
    explicit Checkpoint(const std::string& dir) {
        std::vector<std::string> files;
        const std::string index = dir + "/model.safetensors.index.json";
        if (file_exists(index)) {
            const json::Value v = json::parse(read_text(index));
            for (const auto& kv : v.at("weight_map").obj) {
                const std::string& f = kv.second.string();
                if (std::find(files.begin(), files.end(), f) == files.end()) files.push_back(f);
            }
        } else {
            for (const auto& e : std::filesystem::directory_iterator(dir))
                if (e.path().extension() == ".safetensors") files.push_back(e.path().filename().string());
            std::sort(files.begin(), files.end());
        }
        if (files.empty()) throw std::runtime_error("no .safetensors files in " + dir);
        for (const auto& f : files) map_file(dir + "/" + f);
    }
    ~Checkpoint() {
        for (auto& m : maps_) ::munmap(m.first, m.second);
    }
    Checkpoint(const Checkpoint&) = delete;
    Checkpoint& operator=(const Checkpoint&) = delete;

    const TensorRef& get(const std::string& name, const char* dtype, const std::vector<long long>& shape) const {
        auto it = tensors_.find(name);
        if (it == tensors_.end()) throw std::runtime_error("checkpoint: missing tensor " + name);
        const TensorRef& t = it->second;
        if (t.dtype != dtype) throw std::runtime_error("checkpoint: " + name + " is " + t.dtype + ", expected " + dtype);
        if (t.shape != shape) {
            std::string a, b;
            for (long long d : t.shape) a += std::to_string(d) + " ";
            for (long long d : shape) b += std::to_string(d) + " ";
            throw std::runtime_error("checkpoint: " + name + " has shape [ " + a + "], expected [ " + b + "]");
        }
        return t;
    }

  private:
    std::map<std::string, TensorRef> tensors_;
    std::vector<std::pair<void*, size_t>> maps_;

    void map_file(const std::string& path) {
        const int fd = ::open(path.c_str(), O_RDONLY);
        if (fd < 0) throw std::runtime_error("cannot open " + path);
        struct stat st;
        if (::fstat(fd, &st) != 0) {
            ::close(fd);
            throw std::runtime_error("cannot stat " + path);
        }
        const size_t size = size_t(st.st_size);
        void* p = size ? ::mmap(nullptr, size, PROT_READ, MAP_PRIVATE, fd, 0) : MAP_FAILED;
        ::close(fd);
        if (p == MAP_FAILED) throw std::runtime_error("cannot map " + path);
        maps_.emplace_back(p, size);
        const uint8_t* b = static_cast<const uint8_t*>(p);
        if (size < 8) throw std::runtime_error(path + ": not a safetensors file");
        uint64_t hlen = 0;
        for (int i = 7; i >= 0; --i) hlen = (hlen << 8) | b[i];
        if (hlen > size - 8) throw std::runtime_error(path + ": header past the end of the file");
        const json::Value h = json::parse(std::string(reinterpret_cast<const char*>(b + 8), size_t(hlen)));
        const uint8_t* data = b + 8 + hlen;
        const size_t data_size = size - 8 - size_t(hlen);
        for (const auto& kv : h.obj) {
            if (kv.first == "__metadata__") continue;
            TensorRef t;
            t.dtype = kv.second.at("dtype").string();
            for (const auto& d : kv.second.at("shape").arr) t.shape.push_back(d.integer());
            const auto& off = kv.second.at("data_offsets").arr;
            if (off.size() != 2) throw std::runtime_error(path + ": bad data_offsets for " + kv.first);
            const size_t o0 = size_t(off[0].integer()), o1 = size_t(off[1].integer());
            if (o0 > o1 || o1 > data_size) throw std::runtime_error(path + ": data_offsets out of range for " + kv.first);
            t.data = data + o0;
            t.nbytes = o1 - o0;
            tensors_[kv.first] = t;
        }
    }
};

void require_cfg(bool ok, const std::string& what) {
    if (!ok) throw std::runtime_error("config: " + what);
}

// ---------------------------------------------------------------------------------------------------- KV fill
// Deterministic N(0, 1) fp16 values for benchmarking with a pre-filled cache: a 64-bit mix of (seed, index) gives two
// uniforms, Box-Muller gives the normal.
__device__ __forceinline__ unsigned long long mix64(unsigned long long z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

__global__ void fill_normal_half_kernel(__half* p, size_t n, unsigned long long seed) {
    for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) {
        const unsigned long long r = mix64(seed * 0x100000001B3ull + i);
        const float u1 = (float(uint32_t(r >> 40)) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = float(uint32_t(r & 0xFFFFFFu)) * (1.0f / 16777216.0f);
        const float z = sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
        p[i] = __float2half_rn(z);
    }
}

}  // namespace

// ---------------------------------------------------------------------------------------------------- config
ModelConfig ModelConfig::load(const std::string& dir) {
    const json::Value j = json::parse(read_text(dir + "/config.json"));
    ModelConfig c;
    c.layers = int(j.at("num_hidden_layers").integer());
    c.hidden = int(j.at("hidden_size").integer());
    c.intermediate = int(j.at("intermediate_size").integer());
    c.vocab = int(j.at("vocab_size").integer());
    c.experts = int(j.has("num_local_experts") ? j.at("num_local_experts").integer() : j.at("num_experts").integer());
    c.top_k = int(j.has("num_experts_per_tok") ? j.at("num_experts_per_tok").integer()
                                               : j.at("experts_per_token").integer());
    c.window = int(j.at("sliding_window").integer());
    c.heads = int(j.at("num_attention_heads").integer());
    c.kv_heads = int(j.at("num_key_value_heads").integer());
    c.head_dim = int(j.at("head_dim").integer());
    c.max_positions = j.has("max_position_embeddings") ? int(j.at("max_position_embeddings").integer()) : 131072;
    if (j.has("rms_norm_eps")) c.eps = float(j.at("rms_norm_eps").number());
    if (j.has("swiglu_limit")) c.swiglu_limit = float(j.at("swiglu_limit").number());
    if (j.has("swiglu_alpha")) c.swiglu_alpha = float(j.at("swiglu_alpha").number());
    const json::Value& r = j.has("rope_scaling") ? j.at("rope_scaling") : j.at("rope_parameters");
    const std::string rt = r.has("rope_type") ? r.at("rope_type").string() : r.at("type").string();
    require_cfg(rt == "yarn", "rope_type must be yarn");
    c.rope_theta = j.has("rope_theta") ? j.at("rope_theta").number() : r.at("rope_theta").number();
    c.rope_factor = r.at("factor").number();
    c.rope_original = int(r.at("original_max_position_embeddings").integer());
    c.beta_fast = r.has("beta_fast") ? r.at("beta_fast").number() : 32.0;
    c.beta_slow = r.has("beta_slow") ? r.at("beta_slow").number() : 1.0;
    c.rope_truncate = r.has("truncate") ? r.at("truncate").boolean() : false;
    if (j.has("layer_types"))
        for (const auto& t : j.at("layer_types").arr) c.sliding.push_back(t.string() == "sliding_attention");
    else
        for (int l = 0; l < c.layers; ++l) c.sliding.push_back(l % 2 == 0);
    const std::string gen = dir + "/generation_config.json";
    if (file_exists(gen)) {
        const json::Value g = json::parse(read_text(gen));
        if (g.has("eos_token_id")) {
            const json::Value& e = g.at("eos_token_id");
            if (e.kind == json::Value::Array)
                for (const auto& v : e.arr) c.eos.push_back(int(v.integer()));
            else
                c.eos.push_back(int(e.integer()));
        }
    }
    // The attention kernels are specialised for gpt-oss's geometry; the MoE kernel for its tensor-core shapes.
    require_cfg(c.heads == 64 && c.kv_heads == 8 && c.head_dim == 64, "attention must be 64 heads, 8 kv heads, dim 64");
    require_cfg(int(c.sliding.size()) == c.layers, "layer_types length");
    require_cfg(c.hidden % 64 == 0 && c.intermediate % 64 == 0 && c.hidden <= 3072,
                "hidden and intermediate must be multiples of 64, hidden at most 3072");
    require_cfg(c.experts >= c.top_k && c.experts <= 32 && c.top_k >= 1 && c.top_k <= 8, "1 <= top_k <= 8, top_k <= experts <= 32");
    return c;
}

// ---------------------------------------------------------------------------------------------------- engine
void* Engine::alloc(size_t bytes) {
    if (budget_ > 0 && bytes_ + (long long)bytes > budget_)
        throw std::runtime_error("VRAM budget exceeded: need more than " + std::to_string((bytes_ + bytes) >> 20) +
                                 " MiB, budget " + std::to_string(budget_ >> 20) + " MiB");
    void* p = nullptr;
    GPT_CHECK(cudaMalloc(&p, bytes));
    allocs_.push_back(p);
    bytes_ += (long long)bytes;
    return p;
}

Engine::Engine(const std::string& dir, int max_ctx, long long vram_budget) : cfg_(ModelConfig::load(dir)),
                                                                              budget_(vram_budget) {
    if (max_ctx <= 0 || max_ctx > cfg_.max_positions)
        throw std::runtime_error("max_ctx must be in 1.." + std::to_string(cfg_.max_positions));
    max_ctx_ = max_ctx;
    GPT_CHECK(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking));
    try {
        Checkpoint ck(dir);
        const long long H = cfg_.hidden, I = cfg_.intermediate, E = cfg_.experts, V = cfg_.vocab;
        const long long QD = (long long)cfg_.heads * cfg_.head_dim, KVD = (long long)cfg_.kv_heads * cfg_.head_dim;
        auto put = [&](void* dst, const void* src, size_t n) {
            GPT_CHECK(cudaMemcpy(dst, src, n, cudaMemcpyHostToDevice));
        };
        auto raw = [&](const std::string& n, const char* dtype, const std::vector<long long>& shape) {
            const TensorRef& t = ck.get(n, dtype, shape);
            void* d = alloc(t.nbytes);
            put(d, t.data, t.nbytes);
            return d;
        };
        auto widen = [](const TensorRef& t, std::vector<float>& out) {     // bf16 -> fp32, exact
            const uint16_t* s = reinterpret_cast<const uint16_t*>(t.data);
            const size_t n = t.nbytes / 2, o = out.size();
            out.resize(o + n);
            for (size_t i = 0; i < n; ++i) {
                const uint32_t w = uint32_t(s[i]) << 16;
                std::memcpy(&out[o + i], &w, 4);
            }
        };
        auto f32 = [&](const std::string& n, const std::vector<long long>& shape) {
            std::vector<float> h;
            widen(ck.get(n, "BF16", shape), h);
            float* d = static_cast<float*>(alloc(h.size() * 4));
            put(d, h.data(), h.size() * 4);
            return d;
        };
        embed_ = raw("model.embed_tokens.weight", "BF16", {V, H});
        lm_head_ = raw("lm_head.weight", "BF16", {V, H});
        norm_ = f32("model.norm.weight", {H});
        layers_.resize(size_t(cfg_.layers));
        for (int l = 0; l < cfg_.layers; ++l) {
            Layer& L = layers_[size_t(l)];
            const std::string p = "model.layers." + std::to_string(l) + ".";
            L.window = cfg_.sliding[size_t(l)] ? cfg_.window : 0;
            // Q, K and V rows end to end: one GEMV computes all three
            const TensorRef& q = ck.get(p + "self_attn.q_proj.weight", "BF16", {QD, H});
            const TensorRef& k = ck.get(p + "self_attn.k_proj.weight", "BF16", {KVD, H});
            const TensorRef& v = ck.get(p + "self_attn.v_proj.weight", "BF16", {KVD, H});
            L.wqkv = alloc(q.nbytes + k.nbytes + v.nbytes);
            put(L.wqkv, q.data, q.nbytes);
            put(static_cast<char*>(L.wqkv) + q.nbytes, k.data, k.nbytes);
            put(static_cast<char*>(L.wqkv) + q.nbytes + k.nbytes, v.data, v.nbytes);
            std::vector<float> b;
            widen(ck.get(p + "self_attn.q_proj.bias", "BF16", {QD}), b);
            widen(ck.get(p + "self_attn.k_proj.bias", "BF16", {KVD}), b);
            widen(ck.get(p + "self_attn.v_proj.bias", "BF16", {KVD}), b);
            L.bqkv = static_cast<float*>(alloc(b.size() * 4));
            put(L.bqkv, b.data(), b.size() * 4);
            L.wo = raw(p + "self_attn.o_proj.weight", "BF16", {H, QD});
            L.bo = f32(p + "self_attn.o_proj.bias", {H});
            L.sinks = f32(p + "self_attn.sinks", {cfg_.heads});
            L.ln1 = f32(p + "input_layernorm.weight", {H});
            L.ln2 = f32(p + "post_attention_layernorm.weight", {H});
            L.wr = raw(p + "mlp.router.weight", "BF16", {E, H});
            L.br = f32(p + "mlp.router.bias", {E});
            L.gu_blocks = static_cast<uint8_t*>(raw(p + "mlp.experts.gate_up_proj_blocks", "U8", {E, 2 * I, H / 32, 16}));
            L.gu_scales = static_cast<uint8_t*>(raw(p + "mlp.experts.gate_up_proj_scales", "U8", {E, 2 * I, H / 32}));
            L.gu_bias = f32(p + "mlp.experts.gate_up_proj_bias", {E, 2 * I});
            L.dn_blocks = static_cast<uint8_t*>(raw(p + "mlp.experts.down_proj_blocks", "U8", {E, H, I / 32, 16}));
            L.dn_scales = static_cast<uint8_t*>(raw(p + "mlp.experts.down_proj_scales", "U8", {E, H, I / 32}));
            L.dn_bias = f32(p + "mlp.experts.down_proj_bias", {E, H});
            // the prepared MoE layer (scales repacked once for the tensor cores; refuses E8M0 0xFF scales)
            L.moe = gptoss_moe_layer_create(L.ln2, cfg_.eps, L.wr, L.br, L.gu_blocks, L.gu_scales, L.gu_bias,
                                            L.dn_blocks, L.dn_scales, L.dn_bias, cfg_.experts, cfg_.top_k,
                                            cfg_.hidden, cfg_.intermediate, cfg_.swiglu_alpha, cfg_.swiglu_limit);
            if (!L.moe) throw std::runtime_error(p + "mlp: " + gptoss_last_error());
            L.slots = L.window > 0 ? size_t(L.window) : size_t(max_ctx_);
            L.kc = alloc(L.slots * size_t(KVD) * 2);
            L.vc = alloc(L.slots * size_t(KVD) * 2);
        }

        // YaRN rotary tables (float32 throughout, as gptoss_ref/rope.py computes them): inverse frequencies blended
        // between interpolation (1 / (factor theta^(2i/d))) and extrapolation (1 / theta^(2i/d)) by a linear ramp
        // over the correction range [low, high] of pair indices, angles pos * inv_freq, and cos / sin scaled by the
        // attention concentration 0.1 ln(factor) + 1.
        const int d = cfg_.head_dim, half = d / 2;
        auto dim_for = [&](double rotations) {
            return d * std::log(cfg_.rope_original / (rotations * 2.0 * M_PI)) / (2.0 * std::log(cfg_.rope_theta));
        };
        double low = dim_for(cfg_.beta_fast), high = dim_for(cfg_.beta_slow);
        if (cfg_.rope_truncate) {
            low = std::floor(low);
            high = std::ceil(high);
        }
        low = std::max(low, 0.0);
        high = std::min(high, double(d - 1));
        if (high == low) high += 0.001;
        std::vector<float> inv(static_cast<size_t>(half), 0.0f);
        for (int i = 0; i < half; ++i) {
            const float fr = std::pow(float(cfg_.rope_theta), float(2 * i) / float(d));
            const float extrapolation = 1.0f / fr, interpolation = 1.0f / (float(cfg_.rope_factor) * fr);
            const float ramp = std::min(std::max((float(i) - float(low)) / float(high - low), 0.0f), 1.0f);
            inv[size_t(i)] = interpolation * ramp + extrapolation * (1.0f - ramp);
        }
        const float conc = cfg_.rope_factor > 1.0 ? float(0.1 * std::log(cfg_.rope_factor) + 1.0) : 1.0f;
        std::vector<float> ct(size_t(max_ctx_) * half), st(size_t(max_ctx_) * half);
        for (int pos = 0; pos < max_ctx_; ++pos)
            for (int i = 0; i < half; ++i) {
                const float ang = float(pos) * inv[size_t(i)];
                ct[size_t(pos) * half + i] = std::cos(ang) * conc;
                st[size_t(pos) * half + i] = std::sin(ang) * conc;
            }
        cos_ = static_cast<float*>(alloc(ct.size() * 4));
        sin_ = static_cast<float*>(alloc(st.size() * 4));
        put(cos_, ct.data(), ct.size() * 4);
        put(sin_, st.data(), st.size() * 4);

        x_ = static_cast<float*>(alloc(size_t(H) * 4));
        qkv_ = static_cast<float*>(alloc(size_t(QD + 2 * KVD) * 4));
        attn_ = static_cast<float*>(alloc(size_t(QD) * 4));
        part_ = static_cast<float*>(alloc(attention_workspace_floats() * 4));
        GPT_CHECK(cudaMemset(part_, 0, attention_workspace_floats() * 4));
        logits_ = static_cast<float*>(alloc(size_t(V) * 4));
        score_work_ = alloc(score_workspace_bytes());
        GPT_CHECK(cudaMemset(score_work_, 0, score_workspace_bytes()));
        score_f_ = static_cast<float*>(alloc(size_t(score_cap_ + 2) * 4));
        score_i_ = static_cast<int*>(alloc(size_t(score_cap_ + 1) * 4));
        token_ = static_cast<int*>(alloc(4));
        pos_d_ = static_cast<int*>(alloc(4));
        next_token_ = static_cast<int*>(alloc(4));
        err_ = static_cast<int*>(alloc(16));
        GPT_CHECK(cudaMemset(err_, 0, 16));
        ab_work_ = alloc(attn_block_workspace_bytes());
        GPT_CHECK(cudaMemset(ab_work_, 0, attn_block_workspace_bytes()));
        const size_t ws = moe_layer_workspace_bytes(cfg_.top_k, cfg_.hidden, cfg_.intermediate);
        moe_ws_ = alloc(ws);
        GPT_CHECK(cudaMemset(moe_ws_, 0, ws));
        GPT_CHECK(cudaDeviceSynchronize());
        reset();
    } catch (...) {
        for (Layer& L : layers_)
            if (L.moe) gptoss_moe_layer_destroy(L.moe);
        for (void* p : allocs_) cudaFree(p);
        cudaStreamDestroy(stream_);
        throw;
    }
}

Engine::~Engine() {
    if (graph_) cudaGraphExecDestroy(graph_);
    if (cublas_) cublasDestroy(cublas_);
    if (pinned_) cudaFreeHost(pinned_);
    for (Layer& L : layers_)
        if (L.moe) gptoss_moe_layer_destroy(L.moe);
    for (void* p : allocs_) cudaFree(p);
    if (stream_) cudaStreamDestroy(stream_);
}

void Engine::set_position(int pos) {
    if (pos < 0 || pos > max_ctx_) throw std::runtime_error("position out of range");
    pos_ = pos;
    GPT_CHECK(cudaMemcpyAsync(pos_d_, &pos, sizeof(int), cudaMemcpyHostToDevice, stream_));
    GPT_CHECK(cudaStreamSynchronize(stream_));
}

void Engine::forward(cudaStream_t s, bool pdl) {
    const int H = cfg_.hidden;
    const int QD = cfg_.heads * cfg_.head_dim, KVD = cfg_.kv_heads * cfg_.head_dim;
    launch_embed(embed_, token_, x_, H, s, pdl);
    const bool fused = g_attn_impl.load() == 1;
    for (const Layer& L : layers_) {
        if (!fused || !launch_attn_block(x_, L.ln1, cfg_.eps, L.wqkv, L.bqkv, L.wo, L.bo, cos_, sin_, L.kc, L.vc,
                                         L.sinks, pos_d_, L.window, H, ab_work_, err_, s, pdl)) {
            launch_gemv_bf16(L.wqkv, x_, L.ln1, cfg_.eps, L.bqkv, nullptr, qkv_, QD + 2 * KVD, H, s, pdl);
            launch_attention_step(qkv_, cos_, sin_, L.kc, L.vc, L.sinks, pos_d_, L.window, part_, attn_, s, pdl);
            launch_gemv_bf16(L.wo, attn_, nullptr, 0.f, L.bo, x_, x_, H, QD, s, pdl);
        }
        moe_layer_forward_ws(L.moe, x_, x_, s, nullptr, moe_ws_);
    }
    launch_gemv_bf16(lm_head_, x_, norm_, cfg_.eps, nullptr, nullptr, logits_, cfg_.vocab, H, s, pdl);
    if (greedy_graph_)                                           // the next token of a greedy decode, on device
        launch_score(logits_, cfg_.vocab, score_work_, nullptr, 0, -1, nullptr, nullptr, nullptr, nullptr, token_, s, pdl);
    launch_increment(pos_d_, s, pdl);
}

void Engine::capture() {
    if (graph_) {
        cudaGraphExecDestroy(graph_);
        graph_ = nullptr;
    }
    cudaGraph_t g = nullptr;
    GPT_CHECK(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal));
    try {
        forward(stream_, true);
    } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
    }
    GPT_CHECK(cudaStreamEndCapture(stream_, &g));
    const cudaError_t e = cudaGraphInstantiate(&graph_, g, 0);
    cudaGraphDestroy(g);
    GPT_CHECK(e);
}

// One step with the token already in device memory. The first step runs eagerly (it also sizes the workspaces the
// kernels keep per thread); later ones replay the captured graph when graphs are on.
void Engine::run_step() {
    if (graph_on_ && graph_) {
        GPT_CHECK(cudaGraphLaunch(graph_, stream_));
    } else {
        forward(stream_, false);
        if (graph_on_) {
            GPT_CHECK(cudaStreamSynchronize(stream_));
            capture();
        }
    }
}

void Engine::step(int token) {
    if (token < 0 || token >= cfg_.vocab) throw std::runtime_error("token id out of range");
    if (pos_ >= max_ctx_) throw std::runtime_error("context is full");
    if (greedy_graph_) {                                          // the plain step graph
        greedy_graph_ = false;
        if (graph_) { cudaGraphExecDestroy(graph_); graph_ = nullptr; }
    }
    GPT_CHECK(cudaMemcpyAsync(token_, &token, sizeof(int), cudaMemcpyHostToDevice, stream_));
    run_step();
    ++pos_;
}

void Engine::copy_logits(float* host) {
    GPT_CHECK(cudaMemcpyAsync(host, logits_, size_t(cfg_.vocab) * 4, cudaMemcpyDeviceToHost, stream_));
    GPT_CHECK(cudaStreamSynchronize(stream_));
    check_device_error();
}

// The step kernels' error word (a bounded wait that ran out), read after the stream has been synchronized; on an
// error the attention block's workspace (its barrier word and head counters) is zero-filled again.
void Engine::check_device_error() {
    int e = 0;
    GPT_CHECK(cudaMemcpy(&e, err_, sizeof(int), cudaMemcpyDeviceToHost));
    if (e) {
        GPT_CHECK(cudaMemset(err_, 0, sizeof(int)));
        GPT_CHECK(cudaMemset(ab_work_, 0, attn_block_workspace_bytes()));
        throw std::runtime_error("decode step: a bounded wait in the attention block ran out (code " +
                                 std::to_string(e) + ")");
    }
}

void Engine::score(const int* ids, int k, int target, float* lp, int* argmax, float* target_lp, float* lse) {
    if (k < 0 || k > score_cap_) throw std::runtime_error("score: k out of range");
    if (k > 0 && (!ids || !lp)) throw std::runtime_error("score: ids and lp are required when k > 0");
    if (target >= cfg_.vocab) throw std::runtime_error("score: target out of range");
    for (int i = 0; i < k; ++i)
        if (ids[i] < 0 || ids[i] >= cfg_.vocab) throw std::runtime_error("score: id out of range");
    if (k) GPT_CHECK(cudaMemcpyAsync(score_i_, ids, size_t(k) * 4, cudaMemcpyHostToDevice, stream_));
    launch_score(logits_, cfg_.vocab, score_work_, score_i_, k, target, score_f_, score_i_ + score_cap_,
                 score_f_ + score_cap_, score_f_ + score_cap_ + 1, nullptr, stream_, false);
    if (k) GPT_CHECK(cudaMemcpyAsync(lp, score_f_, size_t(k) * 4, cudaMemcpyDeviceToHost, stream_));
    float tail[2];
    int am = 0;
    GPT_CHECK(cudaMemcpyAsync(tail, score_f_ + score_cap_, sizeof(tail), cudaMemcpyDeviceToHost, stream_));
    GPT_CHECK(cudaMemcpyAsync(&am, score_i_ + score_cap_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    GPT_CHECK(cudaStreamSynchronize(stream_));
    if (argmax) *argmax = am;
    if (target_lp) *target_lp = target >= 0 ? tail[0] : 0.f;
    if (lse) *lse = tail[1];
}

void Engine::prefill_stepwise(const int* tokens, int n, const int* ids, int k, float* lp, int* argmax,
                              float* target_lp) {
    if (n <= 0) throw std::runtime_error("prefill: n must be positive");
    if (pos_ + n > max_ctx_) throw std::runtime_error("context is full");
    for (int p = 0; p < n; ++p) {
        step(tokens[p]);
        if (ids && p + 1 < n)
            score(ids + size_t(p) * k, k, tokens[p + 1], lp + size_t(p) * k, argmax + p, target_lp + p, nullptr);
    }
    GPT_CHECK(cudaStreamSynchronize(stream_));
}

void* Engine::scratch(size_t i, size_t bytes) {
    if (pre_.size() <= i) pre_.resize(i + 1, {nullptr, 0});
    auto& b = pre_[i];
    if (b.second < bytes) {
        if (b.first) {
            GPT_CHECK(cudaFree(b.first));
            bytes_ -= (long long)b.second;
            allocs_.erase(std::find(allocs_.begin(), allocs_.end(), b.first));
            b = {nullptr, 0};
        }
        b.first = alloc(bytes);
        b.second = bytes;
    }
    return b.first;
}

// out[rows][n_out] (= or +=) x W^T for x = hi + lo (bf16 rows, K wide) and W bf16 [n_out][K]: two cuBLAS bf16 GEMMs
// with fp32 accumulation, so the activations keep 16 significant bits while the weights stay as stored.
void Engine::project(const void* W, int n_out, int K, const void* hi, const void* lo, int rows, float* out,
                     bool accumulate) {
    const float one = 1.f, zero = 0.f;
    for (int pass = 0; pass < 2; ++pass) {
        const float* beta = pass == 0 && !accumulate ? &zero : &one;
        const cublasStatus_t st = cublasGemmEx(cublas_, CUBLAS_OP_T, CUBLAS_OP_N, n_out, rows, K, &one, W, CUDA_R_16BF,
                                               K, pass == 0 ? hi : lo, CUDA_R_16BF, K, beta, out, CUDA_R_32F, n_out,
                                               CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
        if (st != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("prefill: cublasGemmEx failed (" + std::to_string(int(st)) + ")");
    }
}

// Batched prefill (gptoss.h: the same distributions as n single steps), layer-major as the fp32 reference runs a
// batch (gptoss_ref/model.py:107-125): per layer, the n rows' QKV projection on tensor cores, RoPE and fp16 rounding
// of the new keys and values, causal attention of every row (sinks, window), the batch appended to the cache, the O
// projection plus residual, and the MoE of all n rows through the batched grouped-GEMM path; then the final norm and
// the LM head for the rows that are scored (tensor cores, in chunks) and for the last row (the decode GEMV, whose
// logits the next step's score and gptoss_logits read).
void Engine::prefill(const int* tokens, int n, const int* ids, int k, float* lp, int* argmax, float* target_lp) {
    if (n <= 0) throw std::runtime_error("prefill: n must be positive");
    if (pos_ + n > max_ctx_) throw std::runtime_error("context is full");
    for (int i = 0; i < n; ++i)
        if (tokens[i] < 0 || tokens[i] >= cfg_.vocab) throw std::runtime_error("prefill: token id out of range");
    if (ids) {
        if (k < 0 || k > score_cap_) throw std::runtime_error("prefill: k out of range");
        for (long long i = 0; i < (long long)(n - 1) * k; ++i)
            if (ids[i] < 0 || ids[i] >= cfg_.vocab) throw std::runtime_error("prefill: id out of range");
    }
    if (n == 1) return prefill_stepwise(tokens, n, ids, k, lp, argmax, target_lp);
    if (greedy_graph_) {                                          // the next step captures the plain step graph
        greedy_graph_ = false;
        if (graph_) { cudaGraphExecDestroy(graph_); graph_ = nullptr; }
    }
    if (!cublas_) {
        if (cublasCreate(&cublas_) != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("prefill: cublasCreate failed");
    }
    if (cublasSetStream(cublas_, stream_) != CUBLAS_STATUS_SUCCESS) throw std::runtime_error("prefill: cublasSetStream");
    const int H = cfg_.hidden, V = cfg_.vocab;
    const int QD = cfg_.heads * cfg_.head_dim, QKV = QD + 2 * cfg_.kv_heads * cfg_.head_dim;
    const int p0 = pos_;
    constexpr int kPartRows = 64, kLogitRows = 32;
    float* X = static_cast<float*>(scratch(0, size_t(n) * H * 4));
    const int Kmax = std::max(H, QD);
    void* hi = scratch(1, size_t(n) * Kmax * 2);
    void* lo = scratch(2, size_t(n) * Kmax * 2);
    float* Q = static_cast<float*>(scratch(3, size_t(n) * QKV * 4));
    void* kvb = scratch(4, size_t(n) * 2 * cfg_.kv_heads * cfg_.head_dim * 2);
    float* A = static_cast<float*>(scratch(5, size_t(n) * QD * 4));
    float* part = static_cast<float*>(scratch(6, prefill_attention_floats(kPartRows) * 4));
    int* tok_d = static_cast<int*>(scratch(7, size_t(n) * 4));
    cudaStream_t s = stream_;
    GPT_CHECK(cudaMemcpyAsync(tok_d, tokens, size_t(n) * 4, cudaMemcpyHostToDevice, s));
    launch_embed_rows(embed_, tok_d, X, n, H, s);
    for (const Layer& L : layers_) {
        launch_split_rows(X, n, H, L.ln1, cfg_.eps, hi, lo, s);
        project(L.wqkv, QKV, H, hi, lo, n, Q, false);
        launch_prefill_qkv_rope(Q, L.bqkv, cos_, sin_, p0, n, kvb, s);
        launch_prefill_attention(Q, kvb, L.kc, L.vc, L.sinks, p0, n, L.window, part, kPartRows, A, s);
        launch_prefill_append(kvb, p0, n, L.window, L.kc, L.vc, s);
        launch_split_rows(A, n, QD, nullptr, 0.f, hi, lo, s);
        project(L.wo, H, QD, hi, lo, n, X, true);
        launch_add_bias_rows(X, L.bo, n, H, s);
        if (gptoss_moe_layer_forward_batched(L.moe, X, X, n, s, nullptr) != 0)
            throw std::runtime_error(std::string("prefill moe: ") + gptoss_last_error());
    }
    if (ids && n > 1) {
        const int rows = n - 1;
        float* LG = static_cast<float*>(scratch(8, size_t(kLogitRows) * V * 4));
        int* ids_d = static_cast<int*>(scratch(9, size_t(rows) * std::max(k, 1) * 4));
        float* lp_d = static_cast<float*>(scratch(10, size_t(rows) * (std::max(k, 0) + 1) * 4));
        int* am_d = static_cast<int*>(scratch(11, size_t(rows) * 4));
        float* tl_d = lp_d + size_t(rows) * k;
        if (k) GPT_CHECK(cudaMemcpyAsync(ids_d, ids, size_t(rows) * k * 4, cudaMemcpyHostToDevice, s));
        for (int c0 = 0; c0 < rows; c0 += kLogitRows) {
            const int rc = std::min(kLogitRows, rows - c0);
            launch_split_rows(X + size_t(c0) * H, rc, H, norm_, cfg_.eps, hi, lo, s);
            project(lm_head_, V, H, hi, lo, rc, LG, false);
            for (int r = 0; r < rc; ++r) {
                const int t = c0 + r;
                launch_score(LG + size_t(r) * V, V, score_work_, ids_d + size_t(t) * k, k, tokens[t + 1],
                             lp_d + size_t(t) * k, am_d + t, tl_d + t, nullptr, nullptr, s, false);
            }
        }
        if (k) GPT_CHECK(cudaMemcpyAsync(lp, lp_d, size_t(rows) * k * 4, cudaMemcpyDeviceToHost, s));
        GPT_CHECK(cudaMemcpyAsync(argmax, am_d, size_t(rows) * 4, cudaMemcpyDeviceToHost, s));
        GPT_CHECK(cudaMemcpyAsync(target_lp, tl_d, size_t(rows) * 4, cudaMemcpyDeviceToHost, s));
    }
    // the last row's logits, through the decode path's LM head
    launch_gemv_bf16(lm_head_, X + size_t(n - 1) * H, norm_, cfg_.eps, nullptr, nullptr, logits_, V, H, s, false);
    GPT_CHECK(cudaStreamSynchronize(s));
    set_position(p0 + n);
}

void Engine::bench_steps(int token, int n) {
    if (token < 0 || token >= cfg_.vocab) throw std::runtime_error("token id out of range");
    if (n < 0 || pos_ + n > max_ctx_) throw std::runtime_error("context is full");
    for (int i = 0; i < n; ++i) step(token);
    GPT_CHECK(cudaStreamSynchronize(stream_));
    check_device_error();
}

// Greedy decode: the argmax of each step's logits is written to the device token the next step embeds, so steps
// follow each other without a host round trip; out_tokens[i] (host) receives the i-th generated token.
void Engine::greedy(int token, int n, int* out_tokens) {
    if (token < 0 || token >= cfg_.vocab) throw std::runtime_error("token id out of range");
    if (n < 0 || pos_ + n > max_ctx_) throw std::runtime_error("context is full");
    if (!greedy_graph_) {
        greedy_graph_ = true;
        if (graph_) { cudaGraphExecDestroy(graph_); graph_ = nullptr; }
    }
    if (pinned_n_ < n) {                                          // grow-only pinned buffer for the tokens
        if (pinned_) GPT_CHECK(cudaFreeHost(pinned_));
        pinned_ = nullptr;
        pinned_n_ = 0;
        GPT_CHECK(cudaMallocHost(&pinned_, size_t(std::max(n, 1)) * sizeof(int)));
        pinned_n_ = n;
    }
    GPT_CHECK(cudaMemcpyAsync(token_, &token, sizeof(int), cudaMemcpyHostToDevice, stream_));
    for (int i = 0; i < n; ++i) {
        run_step();
        ++pos_;
        GPT_CHECK(cudaMemcpyAsync(pinned_ + i, token_, sizeof(int), cudaMemcpyDeviceToHost, stream_));
    }
    GPT_CHECK(cudaStreamSynchronize(stream_));
    check_device_error();
    if (out_tokens) std::memcpy(out_tokens, pinned_, size_t(n) * sizeof(int));
}

void Engine::kv_fill_random(int positions, unsigned long long seed) {
    if (positions < 0 || positions > max_ctx_) throw std::runtime_error("kv_fill_random: positions out of range");
    const size_t KVD = size_t(cfg_.kv_heads) * cfg_.head_dim;
    for (size_t l = 0; l < layers_.size(); ++l) {
        const Layer& L = layers_[l];
        const size_t used = std::min(L.slots, size_t(positions)) * KVD;
        if (!used) continue;
        fill_normal_half_kernel<<<num_sms() * 4, 256, 0, stream_>>>(static_cast<__half*>(L.kc), used, seed * 2654435761ull + 2 * l);
        fill_normal_half_kernel<<<num_sms() * 4, 256, 0, stream_>>>(static_cast<__half*>(L.vc), used, seed * 2654435761ull + 2 * l + 1);
        check_launch("kv_fill_random");
    }
    GPT_CHECK(cudaStreamSynchronize(stream_));
    set_position(positions);
}

}  // namespace gpt
