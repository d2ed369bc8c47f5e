// The decode engine behind the reference runtime's engine entry points (gptoss_create, gptoss_step, gptoss_logits,
// gptoss_score, gptoss_prefill, ...): a gpt-oss checkpoint (config.json + safetensors, Hugging Face names) on one
// GPU, one token per step.
#pragma once
#include <cublas_v2.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "gptoss.h"

namespace gpt {

struct ModelConfig {
    int layers = 0, hidden = 0, intermediate = 0, vocab = 0, experts = 0, top_k = 0, window = 0;
    int heads = 0, kv_heads = 0, head_dim = 0, max_positions = 0;
    float eps = 1e-5f, swiglu_limit = 7.0f, swiglu_alpha = 1.702f;
    double rope_theta = 150000.0, rope_factor = 1.0, beta_fast = 32.0, beta_slow = 1.0;
    int rope_original = 4096;
    bool rope_truncate = false;
    std::vector<bool> sliding;                 // per layer: sliding-window attention
    std::vector<int> eos;
    static ModelConfig load(const std::string& dir);
};

class Engine {
  public:
    Engine(const std::string& dir, int max_ctx, long long vram_budget);
    ~Engine();
    Engine(const Engine&) = delete;
    Engine& operator=(const Engine&) = delete;

    int vocab() const { return cfg_.vocab; }
    int position() const { return pos_; }
    long long device_bytes() const { return bytes_; }
    void reset() { set_position(0); }
    void set_position(int pos);
    void use_graph(bool on) { graph_on_ = on; }
    void step(int token);
    void copy_logits(float* host);
    void score(const int* ids, int k, int target, float* lp, int* argmax, float* target_lp, float* lse);
    void prefill(const int* tokens, int n, const int* ids, int k, float* lp, int* argmax, float* target_lp);
    void bench_steps(int token, int n);
    void greedy(int token, int n, int* out_tokens);
    void kv_fill_random(int positions, unsigned long long seed);
    // n single steps (the reference's prefill) instead of the batched path, for comparisons
    void prefill_stepwise(const int* tokens, int n, const int* ids, int k, float* lp, int* argmax, float* target_lp);

  private:
    struct Layer {
        int window = 0;
        void* wqkv = nullptr;                  // bf16 [QD + 2 KVD][H]
        float* bqkv = nullptr;
        void* wo = nullptr;                    // bf16 [H][QD]
        float *bo = nullptr, *sinks = nullptr, *ln1 = nullptr, *ln2 = nullptr;
        void* wr = nullptr;                    // router bf16 [E][H]
        float* br = nullptr;
        uint8_t *gu_blocks = nullptr, *gu_scales = nullptr, *dn_blocks = nullptr, *dn_scales = nullptr;
        float *gu_bias = nullptr, *dn_bias = nullptr;
        gptoss_moe_layer* moe = nullptr;
        void *kc = nullptr, *vc = nullptr;     // fp16 [slots][kv_heads][head_dim]
        size_t slots = 0;
    };
    void* alloc(size_t bytes);
    void forward(cudaStream_t s, bool pdl);
    void capture();
    void run_step();
    void check_device_error();
    void* scratch(size_t i, size_t bytes);     // grow-only buffers of the batched prefill, counted in device_bytes
    void project(const void* W, int n_out, int K, const void* hi, const void* lo, int rows, float* out, bool accumulate);

    ModelConfig cfg_;
    int max_ctx_ = 0, pos_ = 0;
    long long budget_ = 0, bytes_ = 0;
    std::vector<void*> allocs_;
    cudaStream_t stream_ = nullptr;
    cudaGraphExec_t graph_ = nullptr;
    bool graph_on_ = true, greedy_graph_ = false;
    void* embed_ = nullptr;
    void* lm_head_ = nullptr;
    float* norm_ = nullptr;
    std::vector<Layer> layers_;
    float *cos_ = nullptr, *sin_ = nullptr;
    float *x_ = nullptr, *qkv_ = nullptr, *attn_ = nullptr, *part_ = nullptr, *logits_ = nullptr;
    void* score_work_ = nullptr;
    float* score_f_ = nullptr;                  // [score_cap_] log-probabilities, then target_lp, lse
    int* score_i_ = nullptr;                    // [score_cap_] ids, then argmax
    int *token_ = nullptr, *pos_d_ = nullptr, *next_token_ = nullptr;
    int* err_ = nullptr;                        // error word of the attention block (bounded waits)
    void* ab_work_ = nullptr;                   // the attention block's workspace (zero-filled)
    void* moe_ws_ = nullptr;                    // the MoE kernel's workspace, owned by this engine
    cublasHandle_t cublas_ = nullptr;           // the batched prefill's projections (created at its first use)
    std::vector<std::pair<void*, size_t>> pre_; // batched prefill buffers
    int* pinned_ = nullptr;                     // host tokens of a greedy decode
    int pinned_n_ = 0;
    int score_cap_ = 1 << 16;
};

}  // namespace gpt
