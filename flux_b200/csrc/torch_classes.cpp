// torch.classes.flux.NativeSmolLM2Decode / NativeSmolLM2Prefill over the C ABI
// of libfluxb200.so, with the constructor argument lists and method names of
// the reference's custom classes (native_decode_runtime_torch.cpp:38-79,
// native_prefill_runtime_torch.cpp:5-45), so code that builds the runtime
// objects through torch.classes keeps working unchanged.
//
// Each object owns one runtime handle through a shared pointer; the tensors it
// returns are views of the runtime's stable device buffers whose deleters hold
// that pointer, so a view that outlives its object keeps the memory valid.
// The weight tensors given to the constructor are kept referenced for the
// object's lifetime (the runtime borrows them).
#include <ATen/ATen.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/custom_class.h>
#include <torch/library.h>

#include <memory>
#include <string>
#include <vector>

#include "flux_b200.h"

namespace {

constexpr int64_t kHidden = 576;
constexpr int64_t kInter = 1536;
constexpr int64_t kLayers = FX_SMOLLM2_LAYERS;

void check(fx_status status) {
    TORCH_CHECK(status == FX_OK, fx_last_error());
}

void* current_stream(const at::Device& device) {
    return static_cast<void*>(at::cuda::getCurrentCUDAStream(device.index()).stream());
}

void expect_tensor(const at::Tensor& t, const at::Device& device, at::ScalarType dtype,
                   std::vector<int64_t> shape, const std::string& what, const std::string& prefix) {
    TORCH_CHECK(t.defined() && t.is_cuda() && t.device() == device, prefix, ": ", what,
                " must be a CUDA tensor on the runtime's device");
    TORCH_CHECK(t.scalar_type() == dtype, prefix, ": ", what, " has the wrong dtype");
    TORCH_CHECK(t.is_contiguous(), prefix, ": ", what, " must be contiguous");
    TORCH_CHECK(t.sizes() == at::IntArrayRef(shape), prefix, ": ", what, " has shape ", t.sizes(), ", expected ",
                at::IntArrayRef(shape));
}

// The model description from the reference's constructor arguments.
struct Weights {
    std::vector<at::Tensor> keep;  // borrowed by the runtime: referenced while it lives
    fx_model_desc desc{};
};

Weights model_desc(const at::Tensor& embedding, const std::vector<at::Tensor>& input_norm,
                   const std::vector<at::Tensor>& packed_qkv, const std::vector<at::Tensor>& o_proj,
                   const std::vector<at::Tensor>& post_norm, const std::vector<at::Tensor>& gate_up,
                   const std::vector<at::Tensor>& down, const at::Tensor& final_norm, const at::Tensor& lm_head,
                   const at::Tensor& rope_cos, const at::Tensor& rope_sin, int64_t capacity,
                   const std::vector<double>& epsilons, const std::vector<double>& scales, const std::string& prefix) {
    TORCH_CHECK(embedding.defined() && embedding.is_cuda(), prefix, ": embedding weight must be a CUDA tensor");
    const at::Device device = embedding.device();
    TORCH_CHECK(embedding.dim() == 2 && embedding.size(1) == kHidden, prefix, ": embedding weight must be [vocab, 576]");
    const int64_t vocab = embedding.size(0);
    TORCH_CHECK(capacity > 0, prefix, ": cache capacity must be positive");
    for (const auto* list : {&input_norm, &packed_qkv, &o_proj, &post_norm, &gate_up, &down})
        TORCH_CHECK(static_cast<int64_t>(list->size()) == kLayers, prefix, ": exactly 30 layer tensors are required");
    TORCH_CHECK(static_cast<int64_t>(epsilons.size()) == kLayers && static_cast<int64_t>(scales.size()) == kLayers,
                prefix, ": one epsilon and one attention scale per layer are required");
    Weights w;
    auto keep = [&](const at::Tensor& t, std::vector<int64_t> shape, const char* what) {
        expect_tensor(t, device, at::kFloat, std::move(shape), what, prefix);
        w.keep.push_back(t);
        return static_cast<const float*>(t.data_ptr());
    };
    fx_model_desc& d = w.desc;
    d.device = static_cast<int32_t>(device.index());
    d.vocab = vocab;
    d.capacity = capacity;
    d.embedding = keep(embedding, {vocab, kHidden}, "embedding weight");
    d.final_norm = keep(final_norm, {kHidden}, "final norm weight");
    d.lm_head = keep(lm_head, {vocab, kHidden}, "LM-head weight");
    TORCH_CHECK(rope_cos.dim() == 2 && rope_cos.size(0) >= capacity && rope_cos.size(1) == 64 &&
                    rope_sin.sizes() == rope_cos.sizes(),
                prefix, ": RoPE tables must be [>= capacity, 64]");
    d.rope_cos = keep(rope_cos, {rope_cos.size(0), 64}, "RoPE cosine table");
    d.rope_sin = keep(rope_sin, {rope_sin.size(0), 64}, "RoPE sine table");
    for (int64_t l = 0; l < kLayers; ++l) {
        d.input_norm[l] = keep(input_norm[l], {kHidden}, "layer input norm weight");
        d.packed_qkv[l] = keep(packed_qkv[l], {960, kHidden}, "layer packed QKV weight");
        d.o_proj[l] = keep(o_proj[l], {kHidden, kHidden}, "layer attention output weight");
        d.post_norm[l] = keep(post_norm[l], {kHidden}, "layer post-attention norm weight");
        d.gate_up[l] = keep(gate_up[l], {2 * kInter, kHidden}, "layer gate/up weight");
        d.down[l] = keep(down[l], {kHidden, kInter}, "layer down weight");
        TORCH_CHECK(epsilons[l] > 0.0 && epsilons[l] == epsilons[0], prefix,
                    ": every layer must share one positive RMSNorm epsilon");
        TORCH_CHECK(std::isfinite(scales[l]), prefix, ": every attention scale must be finite");
        d.attention_scale[l] = static_cast<float>(scales[l]);
    }
    d.epsilon = static_cast<float>(epsilons[0]);
    return w;
}

// K/V sources [1, 3, rows >= position, 64] per layer (none when position is 0).
int64_t cache_sources(const std::vector<at::Tensor>& keys, const std::vector<at::Tensor>& values, int64_t position,
                      const at::Device& device, const std::string& prefix, std::vector<const float*>& kp,
                      std::vector<const float*>& vp) {
    if (position == 0 && keys.empty() && values.empty()) return 0;
    TORCH_CHECK(static_cast<int64_t>(keys.size()) == kLayers && static_cast<int64_t>(values.size()) == kLayers, prefix,
                ": one K/V tensor per layer is required");
    int64_t rows = -1;
    for (int64_t l = 0; l < kLayers; ++l) {
        const at::Tensor& k = keys[l];
        const at::Tensor& v = values[l];
        TORCH_CHECK(k.defined() && v.defined() && k.device() == device && v.device() == device &&
                        k.scalar_type() == at::kFloat && v.scalar_type() == at::kFloat && k.is_contiguous() &&
                        v.is_contiguous() && k.dim() == 4 && v.sizes() == k.sizes() && k.size(0) == 1 &&
                        k.size(1) == 3 && k.size(2) >= position && k.size(3) == 64,
                    prefix, ": every K/V source must be contiguous float32 [1, 3, sequence>=position, 64]");
        TORCH_CHECK(rows < 0 || k.size(2) == rows, prefix, ": every K/V source must have the same sequence length");
        rows = k.size(2);
        kp.push_back(static_cast<const float*>(k.data_ptr()));
        vp.push_back(static_cast<const float*>(v.data_ptr()));
    }
    return rows;
}

at::Tensor view(void* ptr, std::vector<int64_t> shape, at::ScalarType dtype, const at::Device& device,
                const std::shared_ptr<void>& owner) {
    auto keep = owner;
    return at::from_blob(
        ptr, shape, [keep](void*) mutable { keep.reset(); }, at::TensorOptions().dtype(dtype).device(device));
}

// ------------------------------------------------------------------ decode

// Tensor views and scalars of one fx_decode (owned or borrowed from a prefill).
struct DecodeState {
    fx_decode* handle = nullptr;
    at::Device device = at::Device(at::kCUDA, 0);
    std::shared_ptr<void> owner;
    fx_decode_buffers buffers{};
    int64_t capacity = 0, vocab = 0;

    void init(fx_decode* h, const at::Device& d, std::shared_ptr<void> o) {
        handle = h;
        device = d;
        owner = std::move(o);
        check(fx_decode_get_buffers(handle, &buffers));
        fx_decode_info info{};
        check(fx_decode_get_info(handle, &info));
        capacity = info.capacity;
        vocab = info.vocab;
    }
    fx_decode_info info() const {
        fx_decode_info i{};
        check(fx_decode_get_info(handle, &i));
        return i;
    }
    int64_t read(int32_t which) const {
        c10::cuda::CUDAGuard guard(device);
        int64_t v = 0;
        check(fx_decode_read_state(handle, which, &v));
        return v;
    }
    at::Tensor replay(const c10::optional<at::Tensor>& token, const std::string& prefix) {
        c10::cuda::CUDAGuard guard(device);
        const int64_t* t = nullptr;
        if (token.has_value() && token->defined()) {
            expect_tensor(*token, device, at::kLong, {1, 1}, "replay token", prefix);
            t = token->data_ptr<int64_t>();
        }
        check(fx_decode_replay(handle, t, current_stream(device)));
        return logits();
    }
    at::Tensor generate(int64_t steps) {
        c10::cuda::CUDAGuard guard(device);
        check(fx_decode_set_eos(handle, -1));
        check(fx_decode_generate(handle, steps, current_stream(device)));
        return generated_tokens();
    }
    at::Tensor logits() const { return view(buffers.logits, {1, 1, vocab}, at::kFloat, device, owner); }
    at::Tensor current_token() const { return view(buffers.input_token, {1, 1}, at::kLong, device, owner); }
    at::Tensor generated_tokens() const { return view(buffers.generated_tokens, {capacity}, at::kLong, device, owner); }
    at::Tensor device_generation_step() const { return view(buffers.generation_step, {}, at::kLong, device, owner); }
    at::Tensor key_cache() const {
        return view(buffers.key_cache, {kLayers, 1, 3, capacity, 64}, at::kFloat, device, owner);
    }
    at::Tensor value_cache() const {
        return view(buffers.value_cache, {kLayers, 1, 3, capacity, 64}, at::kFloat, device, owner);
    }
    at::Tensor device_position() const { return view(buffers.position, {}, at::kLong, device, owner); }
    at::Tensor device_cache_length() const { return view(buffers.cache_length, {}, at::kLong, device, owner); }
    at::Tensor workspace() const {
        return view(buffers.workspace, {buffers.workspace_bytes}, at::kByte, device, owner);
    }
    std::vector<int64_t> addresses() const {
        const fx_decode_buffers& b = buffers;
        std::vector<int64_t> out;
        for (const void* p : {static_cast<const void*>(b.input_token), static_cast<const void*>(b.logits),
                              static_cast<const void*>(b.generated_tokens), static_cast<const void*>(b.generation_step),
                              static_cast<const void*>(b.key_cache), static_cast<const void*>(b.value_cache),
                              static_cast<const void*>(b.position), static_cast<const void*>(b.cache_length),
                              static_cast<const void*>(b.workspace), static_cast<const void*>(b.hidden_a),
                              static_cast<const void*>(b.hidden_b), static_cast<const void*>(b.final_norm_output),
                              static_cast<const void*>(b.attention_workspace)})
            out.push_back(static_cast<int64_t>(reinterpret_cast<uintptr_t>(p)));
        return out;
    }
};

class NativeSmolLM2Decode final : public torch::CustomClassHolder {
public:
    NativeSmolLM2Decode(at::Tensor initial_token, at::Tensor embedding_weight,
                        std::vector<at::Tensor> input_norm_weights, std::vector<at::Tensor> packed_qkv_weights,
                        std::vector<at::Tensor> attention_output_weights,
                        std::vector<at::Tensor> post_attention_norm_weights,
                        std::vector<at::Tensor> packed_gate_up_weights,
                        std::vector<at::Tensor> down_projection_weights, at::Tensor final_norm_weight,
                        at::Tensor lm_head_weight, at::Tensor rope_cos, at::Tensor rope_sin,
                        std::vector<at::Tensor> initial_key_caches, std::vector<at::Tensor> initial_value_caches,
                        int64_t cache_capacity, int64_t initial_position, std::vector<double> epsilons,
                        std::vector<double> attention_scales) {
        Weights w = model_desc(embedding_weight, input_norm_weights, packed_qkv_weights, attention_output_weights,
                               post_attention_norm_weights, packed_gate_up_weights, down_projection_weights,
                               final_norm_weight, lm_head_weight, rope_cos, rope_sin, cache_capacity, epsilons,
                               attention_scales, kPrefix);
        const at::Device device = embedding_weight.device();
        expect_tensor(initial_token, device, at::kLong, {1, 1}, "initial token", kPrefix);
        TORCH_CHECK(initial_position >= 0 && initial_position < cache_capacity, kPrefix,
                    ": initial position must be inside capacity");
        std::vector<const float*> kp, vp;
        const int64_t rows =
            cache_sources(initial_key_caches, initial_value_caches, initial_position, device, kPrefix, kp, vp);
        c10::cuda::CUDAGuard guard(device);
        fx_decode* handle = nullptr;
        check(fx_decode_create(&w.desc, initial_token.data_ptr<int64_t>(), kp.empty() ? nullptr : kp.data(),
                               vp.empty() ? nullptr : vp.data(), rows, initial_position, current_stream(device),
                               &handle));
        auto weights = std::make_shared<std::vector<at::Tensor>>(std::move(w.keep));
        std::shared_ptr<void> owner(handle, [weights](void* p) { fx_decode_destroy(static_cast<fx_decode*>(p)); });
        state_.init(handle, device, owner);
    }

    at::Tensor replay(const c10::optional<at::Tensor>& token) { return state_.replay(token, kPrefix); }
    at::Tensor generate_greedy(int64_t decode_steps) { return state_.generate(decode_steps); }
    void reset(const at::Tensor& token, const std::vector<at::Tensor>& key_caches,
               const std::vector<at::Tensor>& value_caches, int64_t position) {
        expect_tensor(token, state_.device, at::kLong, {1, 1}, "token", kPrefix);
        TORCH_CHECK(position >= 0 && position < state_.capacity, kPrefix, ": reset position must be inside capacity");
        std::vector<const float*> kp, vp;
        const int64_t rows = cache_sources(key_caches, value_caches, position, state_.device, kPrefix, kp, vp);
        c10::cuda::CUDAGuard guard(state_.device);
        check(fx_decode_reset(state_.handle, token.data_ptr<int64_t>(), kp.empty() ? nullptr : kp.data(),
                              vp.empty() ? nullptr : vp.data(), rows, position, current_stream(state_.device)));
    }
    at::Tensor logits() const { return state_.logits(); }
    at::Tensor current_token() const { return state_.current_token(); }
    at::Tensor generated_tokens() const { return state_.generated_tokens(); }
    at::Tensor device_generation_step() const { return state_.device_generation_step(); }
    at::Tensor key_cache() const { return state_.key_cache(); }
    at::Tensor value_cache() const { return state_.value_cache(); }
    at::Tensor device_position() const { return state_.device_position(); }
    at::Tensor device_cache_length() const { return state_.device_cache_length(); }
    at::Tensor workspace() const { return state_.workspace(); }
    std::vector<int64_t> addresses() const { return state_.addresses(); }
    int64_t position() { return state_.read(FX_STATE_POSITION); }
    int64_t cache_length() { return state_.read(FX_STATE_CACHE_LENGTH); }
    int64_t capacity() const { return state_.capacity; }
    int64_t replay_count() const { return state_.info().replay_count; }
    int64_t generation_step() { return state_.read(FX_STATE_GENERATION_STEP); }
    int64_t workspace_bytes() const { return state_.buffers.workspace_bytes; }
    int64_t stable_buffer_bytes() const { return state_.buffers.stable_buffer_bytes; }
    int64_t vocabulary_size() const { return state_.vocab; }
    int64_t layer_count() const { return kLayers; }

private:
    static constexpr const char* kPrefix = "flux native full decode";
    DecodeState state_;
};

// ----------------------------------------------------------------- prefill

class NativeSmolLM2Prefill final : public torch::CustomClassHolder {
public:
    NativeSmolLM2Prefill(at::Tensor input_ids, at::Tensor embedding_weight, std::vector<at::Tensor> input_norm_weights,
                         std::vector<at::Tensor> packed_qkv_weights, std::vector<at::Tensor> attention_output_weights,
                         std::vector<at::Tensor> post_attention_norm_weights,
                         std::vector<at::Tensor> packed_gate_up_weights,
                         std::vector<at::Tensor> down_projection_weights, at::Tensor final_norm_weight,
                         at::Tensor lm_head_weight, at::Tensor rope_cos, at::Tensor rope_sin, int64_t cache_capacity,
                         std::vector<double> epsilons, std::vector<double> attention_scales) {
        Weights w = model_desc(embedding_weight, input_norm_weights, packed_qkv_weights, attention_output_weights,
                               post_attention_norm_weights, packed_gate_up_weights, down_projection_weights,
                               final_norm_weight, lm_head_weight, rope_cos, rope_sin, cache_capacity, epsilons,
                               attention_scales, kPrefix);
        const at::Device device = embedding_weight.device();
        TORCH_CHECK(input_ids.defined() && input_ids.dim() == 2 && input_ids.size(0) == 1 && input_ids.size(1) > 0,
                    kPrefix, ": input_ids must be [1, prompt] with a non-empty prompt");
        expect_tensor(input_ids, device, at::kLong, {1, input_ids.size(1)}, "input_ids", kPrefix);
        TORCH_CHECK(input_ids.size(1) <= cache_capacity, kPrefix, ": prompt exceeds fixed cache capacity");
        c10::cuda::CUDAGuard guard(device);
        fx_prefill* handle = nullptr;
        check(fx_prefill_create(&w.desc, input_ids.data_ptr<int64_t>(), input_ids.size(1), current_stream(device),
                                &handle));
        auto weights = std::make_shared<std::vector<at::Tensor>>(std::move(w.keep));
        std::shared_ptr<void> owner(handle, [weights](void* p) { fx_prefill_destroy(static_cast<fx_prefill*>(p)); });
        prefill_ = handle;
        rows_ = fx_prefill_prompt_length(handle);
        check(fx_prefill_get_buffers(handle, &buffers_));
        decode_.init(fx_prefill_decode(handle), device, owner);
    }

    at::Tensor prefill(const at::Tensor& input_ids) {
        expect_tensor(input_ids, decode_.device, at::kLong, {1, rows_}, "input_ids", kPrefix);
        c10::cuda::CUDAGuard guard(decode_.device);
        check(fx_prefill_run(prefill_, input_ids.data_ptr<int64_t>(), current_stream(decode_.device)));
        return logits();
    }
    at::Tensor replay(const c10::optional<at::Tensor>& token) { return decode_.replay(token, kPrefix); }
    // The prefill sampled the first token; max_new_tokens - 1 decode steps add the rest.
    at::Tensor generate_greedy(int64_t max_new_tokens) {
        TORCH_CHECK(max_new_tokens >= 1, kPrefix, ": max_new_tokens must be positive");
        TORCH_CHECK(max_new_tokens <= decode_.capacity - rows_ + 1, kPrefix,
                    ": generation exceeds fixed cache capacity");
        return decode_.generate(max_new_tokens - 1).narrow(0, 0, max_new_tokens).view({1, max_new_tokens});
    }
    at::Tensor logits() const { return view(buffers_.prefill_logits, {1, 1, decode_.vocab}, at::kFloat, decode_.device, decode_.owner); }
    at::Tensor final_hidden() const { return view(buffers_.final_hidden, {1, 1, kHidden}, at::kFloat, decode_.device, decode_.owner); }
    at::Tensor current_token() const { return decode_.current_token(); }
    at::Tensor generated_tokens() const { return decode_.generated_tokens(); }
    at::Tensor device_generation_step() const { return decode_.device_generation_step(); }
    at::Tensor key_cache() const { return decode_.key_cache(); }
    at::Tensor value_cache() const { return decode_.value_cache(); }
    at::Tensor device_position() const { return decode_.device_position(); }
    at::Tensor device_cache_length() const { return decode_.device_cache_length(); }
    std::vector<int64_t> addresses() const {
        std::vector<int64_t> out;
        for (const void* p : {static_cast<const void*>(buffers_.prefill_logits), static_cast<const void*>(buffers_.workspace),
                              static_cast<const void*>(buffers_.attention_output),
                              static_cast<const void*>(buffers_.final_hidden)})
            out.push_back(static_cast<int64_t>(reinterpret_cast<uintptr_t>(p)));
        for (int64_t a : decode_.addresses()) out.push_back(a);
        return out;
    }
    int64_t position() { return decode_.read(FX_STATE_POSITION); }
    int64_t cache_length() { return decode_.read(FX_STATE_CACHE_LENGTH); }
    int64_t prompt_length() const { return rows_; }
    int64_t capacity() const { return decode_.capacity; }
    int64_t replay_count() const { return decode_.info().replay_count; }
    int64_t generation_step() { return decode_.read(FX_STATE_GENERATION_STEP); }
    int64_t workspace_bytes() const { return buffers_.workspace_bytes; }
    int64_t cache_bytes() const { return 2 * kLayers * 3 * decode_.capacity * 64 * 4; }
    int64_t stable_buffer_bytes() const {
        return 8 + decode_.vocab * 4 + decode_.buffers.stable_buffer_bytes;
    }

private:
    static constexpr const char* kPrefix = "flux native prefill";
    fx_prefill* prefill_ = nullptr;
    int64_t rows_ = 0;
    fx_prefill_buffers buffers_{};
    DecodeState decode_;
};

}  // namespace

TORCH_LIBRARY_FRAGMENT(flux, library) {
    library.class_<NativeSmolLM2Decode>("NativeSmolLM2Decode")
        .def(torch::init<at::Tensor, at::Tensor, std::vector<at::Tensor>, std::vector<at::Tensor>,
                         std::vector<at::Tensor>, std::vector<at::Tensor>, std::vector<at::Tensor>,
                         std::vector<at::Tensor>, at::Tensor, at::Tensor, at::Tensor, at::Tensor,
                         std::vector<at::Tensor>, std::vector<at::Tensor>, int64_t, int64_t, std::vector<double>,
                         std::vector<double>>())
        .def("replay", &NativeSmolLM2Decode::replay)
        .def("generate_greedy", &NativeSmolLM2Decode::generate_greedy)
        .def("reset", &NativeSmolLM2Decode::reset)
        .def("logits", &NativeSmolLM2Decode::logits)
        .def("current_token", &NativeSmolLM2Decode::current_token)
        .def("generated_tokens", &NativeSmolLM2Decode::generated_tokens)
        .def("device_generation_step", &NativeSmolLM2Decode::device_generation_step)
        .def("key_cache", &NativeSmolLM2Decode::key_cache)
        .def("value_cache", &NativeSmolLM2Decode::value_cache)
        .def("device_position", &NativeSmolLM2Decode::device_position)
        .def("device_cache_length", &NativeSmolLM2Decode::device_cache_length)
        .def("workspace", &NativeSmolLM2Decode::workspace)
        .def("addresses", &NativeSmolLM2Decode::addresses)
        .def("position", &NativeSmolLM2Decode::position)
        .def("cache_length", &NativeSmolLM2Decode::cache_length)
        .def("capacity", &NativeSmolLM2Decode::capacity)
        .def("replay_count", &NativeSmolLM2Decode::replay_count)
        .def("generation_step", &NativeSmolLM2Decode::generation_step)
        .def("workspace_bytes", &NativeSmolLM2Decode::workspace_bytes)
        .def("stable_buffer_bytes", &NativeSmolLM2Decode::stable_buffer_bytes)
        .def("vocabulary_size", &NativeSmolLM2Decode::vocabulary_size)
        .def("layer_count", &NativeSmolLM2Decode::layer_count);
    library.class_<NativeSmolLM2Prefill>("NativeSmolLM2Prefill")
        .def(torch::init<at::Tensor, at::Tensor, std::vector<at::Tensor>, std::vector<at::Tensor>,
                         std::vector<at::Tensor>, std::vector<at::Tensor>, std::vector<at::Tensor>,
                         std::vector<at::Tensor>, at::Tensor, at::Tensor, at::Tensor, at::Tensor, int64_t,
                         std::vector<double>, std::vector<double>>())
        .def("prefill", &NativeSmolLM2Prefill::prefill)
        .def("replay", &NativeSmolLM2Prefill::replay)
        .def("generate_greedy", &NativeSmolLM2Prefill::generate_greedy)
        .def("logits", &NativeSmolLM2Prefill::logits)
        .def("current_token", &NativeSmolLM2Prefill::current_token)
        .def("generated_tokens", &NativeSmolLM2Prefill::generated_tokens)
        .def("device_generation_step", &NativeSmolLM2Prefill::device_generation_step)
        .def("final_hidden", &NativeSmolLM2Prefill::final_hidden)
        .def("key_cache", &NativeSmolLM2Prefill::key_cache)
        .def("value_cache", &NativeSmolLM2Prefill::value_cache)
        .def("device_position", &NativeSmolLM2Prefill::device_position)
        .def("device_cache_length", &NativeSmolLM2Prefill::device_cache_length)
        .def("addresses", &NativeSmolLM2Prefill::addresses)
        .def("position", &NativeSmolLM2Prefill::position)
        .def("cache_length", &NativeSmolLM2Prefill::cache_length)
        .def("prompt_length", &NativeSmolLM2Prefill::prompt_length)
        .def("capacity", &NativeSmolLM2Prefill::capacity)
        .def("replay_count", &NativeSmolLM2Prefill::replay_count)
        .def("generation_step", &NativeSmolLM2Prefill::generation_step)
        .def("workspace_bytes", &NativeSmolLM2Prefill::workspace_bytes)
        .def("cache_bytes", &NativeSmolLM2Prefill::cache_bytes)
        .def("stable_buffer_bytes", &NativeSmolLM2Prefill::stable_buffer_bytes);
}
