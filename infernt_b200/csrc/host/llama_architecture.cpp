// llama_architecture.cpp — LlamaArchitecture over the fused decode plan.
// The reference's forward (architectures/llama/llama_model.cpp:45-65 and
// llama_layer.cpp:5-73: ~400 launches, 23 blocking copies) becomes one
// launch of the persistent decode kernel (or one graph replay) of the plan
// bound to these weights and this KV cache.
#include <cstdlib>
#include <stdexcept>
#include <string>

#include "architecture.h"

namespace {
void check(int status, const char* what) {
    if (status != INFERNT_OK)
        throw std::runtime_error(std::string(what) + ": " + infernt_status_string(status) + " (" +
                                 infernt_last_error() + ")");
}

const void* ptr(const Tensor& t, const char* name, DType want) {
    if (!t.is_valid() || !t.is_cuda()) throw std::runtime_error(std::string("weight ") + name + " is not a CUDA tensor");
    if (t.dtype() != want)
        throw std::runtime_error(std::string("weight ") + name + " has dtype " + dtype_name(t.dtype()) + ", expected " +
                                 dtype_name(want));
    return t.data_ptr();
}
}  // namespace

namespace {
// INFERNT_DECODE_MODE = eager | graph | persistent (default persistent).
int default_mode() {
    const char* m = std::getenv("INFERNT_DECODE_MODE");
    if (!m) return INFERNT_MODE_PERSISTENT;
    const std::string s(m);
    if (s == "eager") return INFERNT_MODE_EAGER;
    if (s == "graph") return INFERNT_MODE_GRAPH;
    return INFERNT_MODE_PERSISTENT;
}
}  // namespace

LlamaArchitecture::LlamaArchitecture(CublasWrapper& cublas)
    : cublas_(cublas), max_batch_size_(1), mode_(default_mode()), plan_(nullptr) {}

void LlamaArchitecture::set_decode_mode(int mode) {
    if (mode < INFERNT_MODE_EAGER || mode > INFERNT_MODE_PERSISTENT)
        throw std::invalid_argument("set_decode_mode: unknown mode");
    mode_ = mode;
    infernt_plan_destroy(plan_);
    plan_ = nullptr;
    bound_weights_.clear();
}

int LlamaArchitecture::decode_mode() const { return plan_ ? infernt_plan_mode(plan_) : mode_; }

LlamaArchitecture::~LlamaArchitecture() { infernt_plan_destroy(plan_); }

void LlamaArchitecture::allocate_activations(const ModelConfig& config, int max_batch_size) {
    if (max_batch_size != 1)
        throw std::invalid_argument("LlamaArchitecture decodes one sequence (max_batch_size must be 1)");
    config.validate();
    config_ = config;
    max_batch_size_ = max_batch_size;
    infernt_plan_destroy(plan_);
    plan_ = nullptr;
    bound_weights_.clear();
}

infernt_plan* LlamaArchitecture::bind(const ModelWeights& w, KVCache& kv, bool token_input) {
    const ModelConfig& c = config_;
    if (c.num_layers <= 0) throw std::runtime_error("LlamaArchitecture: allocate_activations was not called");
    if ((int)w.layers.size() != c.num_layers || (int)kv.k_cache.size() != c.num_layers ||
        (int)kv.v_cache.size() != c.num_layers)
        throw std::runtime_error("LlamaArchitecture: weights / KV cache layer count mismatch");
    const DType wd = c.weight_dtype;
    std::vector<const void*> wp;
    wp.reserve(3 + 9 * c.num_layers);
    // forward() takes the input embedding and never reads the table (the
    // reference's forward does not either): a caller may leave it empty, and
    // the plan gets the final norm's address as a stand-in it does not read
    const void* fnorm = ptr(w.final_norm, "final_norm", DType::FP32);
    wp.push_back(!token_input && !w.embedding.is_valid() ? fnorm : ptr(w.embedding, "embedding", DType::FP32));
    wp.push_back(fnorm);
    wp.push_back(ptr(w.lm_head, "lm_head", wd));
    for (const auto& lw : w.layers) {
        wp.push_back(ptr(lw.attn_norm, "attn_norm", DType::FP32));
        wp.push_back(ptr(lw.q_proj, "q_proj", wd));
        wp.push_back(ptr(lw.k_proj, "k_proj", wd));
        wp.push_back(ptr(lw.v_proj, "v_proj", wd));
        wp.push_back(ptr(lw.o_proj, "o_proj", wd));
        wp.push_back(ptr(lw.ffn_norm, "ffn_norm", DType::FP32));
        wp.push_back(ptr(lw.gate_proj, "gate_proj", wd));
        wp.push_back(ptr(lw.up_proj, "up_proj", wd));
        wp.push_back(ptr(lw.down_proj, "down_proj", wd));
    }
    std::vector<float*> kp, vp;
    for (int l = 0; l < c.num_layers; ++l) {
        kp.push_back(kv.k_cache[l].data_as_float());
        vp.push_back(kv.v_cache[l].data_as_float());
    }
    if (plan_ && wp == bound_weights_ && kp == bound_k_ && vp == bound_v_) return plan_;
    infernt_plan_destroy(plan_);
    plan_ = nullptr;
    infernt_llama_config pc;
    pc.vocab_size = c.vocab_size;
    pc.hidden_size = c.hidden_size;
    pc.num_layers = c.num_layers;
    pc.num_attention_heads = c.num_attention_heads;
    pc.num_key_value_heads = c.num_key_value_heads;
    pc.intermediate_size = c.intermediate_size;
    pc.max_seq_len = c.max_seq_len;
    pc.head_dim = c.head_dim;
    pc.rms_norm_eps = c.rms_norm_eps;
    pc.rope_theta = c.rope_theta;
    pc.weight_dtype = wd == DType::BF16 ? INFERNT_DTYPE_BF16 : INFERNT_DTYPE_F32;
    check(infernt_plan_create(&pc, wp.data(), kp.data(), vp.data(), mode_, &plan_), "infernt_plan_create");
    bound_weights_ = wp;
    bound_k_ = kp;
    bound_v_ = vp;
    return plan_;
}

void LlamaArchitecture::forward(const Tensor& input, const ModelWeights& w, KVCache& kv, int position,
                                Tensor& logits) {
    infernt_plan* p = bind(w, kv, false);
    if (input.num_elements() != config_.hidden_size || logits.num_elements() != config_.vocab_size)
        throw std::runtime_error("LlamaArchitecture::forward: input or logits shape mismatch");
    check(infernt_plan_forward(p, input.data_as_float(), position, logits.data_as_float(), stream()),
          "LlamaArchitecture::forward");
}

void LlamaArchitecture::forward_token(int token_id, const ModelWeights& w, KVCache& kv, int position,
                                      Tensor& logits) {
    infernt_plan* p = bind(w, kv, true);
    if (logits.num_elements() != config_.vocab_size)
        throw std::runtime_error("LlamaArchitecture::forward_token: logits shape mismatch");
    check(infernt_plan_decode(p, token_id, position, logits.data_as_float(), stream()),
          "LlamaArchitecture::forward_token");
}

void LlamaArchitecture::decode_chain(int token_id, int position, int steps, const ModelWeights& w, KVCache& kv,
                                     int* tokens_dev) {
    infernt_plan* p = bind(w, kv, true);
    check(infernt_plan_decode_chain(p, token_id, position, steps, tokens_dev, stream()),
          "LlamaArchitecture::decode_chain");
}

int LlamaArchitecture::last_token() {
    if (!plan_) throw std::runtime_error("LlamaArchitecture::last_token: no step has run");
    int t = 0;
    check(infernt_plan_read_token(plan_, &t, stream()), "LlamaArchitecture::last_token");
    return t;
}

cudaStream_t LlamaArchitecture::stream() const { return cublas_.stream(); }

int LlamaArchitecture::kernels_per_step() const {
    return plan_ ? infernt_plan_kernels_per_step(plan_) : 5 * config_.num_layers + 1;
}
