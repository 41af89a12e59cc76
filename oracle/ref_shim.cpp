// ref_shim.cpp -- drives tt-lab's own CPU MoE code on caller-supplied buffers.
//
// TEST INFRASTRUCTURE ONLY.  Built by oracle/Makefile together with the
// reference's unmodified src/tensor.cpp, src/gguf.cpp and src/model.cpp (compiled
// from where they lie, with the reference's flags) into oracle/_ref/libttlref.so.
// It lets the parity tests and the benchmark's CPU-baseline leg call exactly the
// reference's GptOssModel::moe (src/model.cpp:292-338) and moe_batch
// (src/model.cpp:340-461) on the same inputs the GPU path sees.
//
// How: GptOssModel needs a GgufFile.  We write a GGUF v3 file that holds only the
// gpt-oss metadata (src/model.cpp:68-98) and a tensor directory in which every
// tensor starts at data offset 0; the file is extended sparsely to the largest
// tensor so the reader's bounds checks (src/gguf.cpp:229-238) pass without disk
// use.  After construction, the data pointers of layer 0's MoE tensors are aimed
// at the caller's buffers.  The model reads nothing else on the MoE path.
// Private members are reached with the explicit-instantiation access idiom
// (access checks do not apply to template arguments of an explicit
// instantiation), which leaves the reference sources untouched.
#include <algorithm>
#include <atomic>
#include <array>
#include <cmath>
#include <limits>
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <initializer_list>
#include <latch>
#include <memory>
#include <stdexcept>
#include <string>
#include <string_view>
#include <thread>
#include <unordered_map>
#include <vector>

#include <fcntl.h>
#include <unistd.h>

#include "gguf.h"
#include "model.h"
#include "tensor.h"

namespace {

template <class Tag, auto Member> struct Expose {
    friend auto member(Tag) {
        return Member;
    }
};

struct TagMoe {
    friend auto member(TagMoe);
};
struct TagMoeBatch {
    friend auto member(TagMoeBatch);
};
struct TagLayers {
    friend auto member(TagLayers);
};
struct TagIndices {
    friend auto member(TagIndices);
};
struct TagWeights {
    friend auto member(TagWeights);
};
struct TagIndicesSeq {
    friend auto member(TagIndicesSeq);
};
struct TagWeightsSeq {
    friend auto member(TagWeightsSeq);
};
struct TagTensors {
    friend auto member(TagTensors);
};
struct TagRouter {
    friend auto member(TagRouter);
};
struct TagRope {
    friend auto member(TagRope);
};
struct TagStoreKv {
    friend auto member(TagStoreKv);
};
struct TagAttend {
    friend auto member(TagAttend);
};

} // namespace

template struct Expose<TagMoe, &GptOssModel::moe>;
template struct Expose<TagMoeBatch, &GptOssModel::moe_batch>;
template struct Expose<TagLayers, &GptOssModel::layers_>;
template struct Expose<TagIndices, &GptOssModel::expert_indices_>;
template struct Expose<TagWeights, &GptOssModel::expert_weights_>;
template struct Expose<TagIndicesSeq, &GptOssModel::expert_indices_sequence_>;
template struct Expose<TagWeightsSeq, &GptOssModel::expert_weights_sequence_>;
template struct Expose<TagTensors, &GgufFile::tensors_>;
template struct Expose<TagRouter, &GptOssModel::router_>;
template struct Expose<TagRope, &GptOssModel::apply_rope>;
template struct Expose<TagStoreKv, &GptOssModel::store_kv>;
template struct Expose<TagAttend, &GptOssModel::attention_from_cache>;

namespace {

constexpr size_t kDim = 2880;

thread_local std::string g_error;

void put(std::string &out, const void *data, size_t size) {
    out.append((const char *)data, size);
}
void put_u32(std::string &out, uint32_t v) {
    put(out, &v, 4);
}
void put_u64(std::string &out, uint64_t v) {
    put(out, &v, 8);
}
void put_str(std::string &out, std::string_view s) {
    put_u64(out, s.size());
    out.append(s);
}
void key_u32(std::string &out, std::string_view key, uint32_t v) {
    put_str(out, key);
    put_u32(out, 4); // GgufType::u32 (src/gguf.h:13-26)
    put_u32(out, v);
}
void key_f32(std::string &out, std::string_view key, float v) {
    put_str(out, key);
    put_u32(out, 6); // GgufType::f32
    put(out, &v, 4);
}
void key_str(std::string &out, std::string_view key, std::string_view v) {
    put_str(out, key);
    put_u32(out, 8); // GgufType::string
    put_str(out, v);
}

struct TensorDef {
    std::string name;
    std::vector<uint64_t> shape;
    uint32_t type;
};

uint64_t def_bytes(const TensorDef &t) {
    uint64_t rows = 1;
    for (size_t i = 1; i < t.shape.size(); ++i) {
        rows *= t.shape[i];
    }
    const uint64_t n = t.shape[0];
    switch (t.type) {
        case tensor_f32:
            return rows * n * 4;
        case tensor_q8_0:
            return rows * n / 32 * 34;
        default:
            return rows * n / 32 * 17;
    }
}

// Writes the metadata-only gpt-oss GGUF for `experts` experts and `layers`
// layers (24 or 36, the two counts GptOssModel accepts, src/model.cpp:71-74).
std::string write_fixture(size_t experts, size_t layers = 24) {
    std::vector<TensorDef> defs;
    defs.push_back({"token_embd.weight", {kDim, 201088}, tensor_q8_0});
    defs.push_back({"output_norm.weight", {kDim}, tensor_f32});
    defs.push_back({"output.weight", {kDim, 201088}, tensor_q8_0});
    for (size_t i = 0; i < layers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        defs.push_back({p + "attn_norm.weight", {kDim}, tensor_f32});
        defs.push_back({p + "post_attention_norm.weight", {kDim}, tensor_f32});
        defs.push_back({p + "attn_q.weight", {kDim, 4096}, tensor_q8_0});
        defs.push_back({p + "attn_q.bias", {4096}, tensor_f32});
        defs.push_back({p + "attn_k.weight", {kDim, 512}, tensor_q8_0});
        defs.push_back({p + "attn_k.bias", {512}, tensor_f32});
        defs.push_back({p + "attn_v.weight", {kDim, 512}, tensor_q8_0});
        defs.push_back({p + "attn_v.bias", {512}, tensor_f32});
        defs.push_back({p + "attn_output.weight", {4096, kDim}, tensor_q8_0});
        defs.push_back({p + "attn_output.bias", {kDim}, tensor_f32});
        defs.push_back({p + "attn_sinks.weight", {64}, tensor_f32});
        defs.push_back({p + "ffn_gate_inp.weight", {kDim, experts}, tensor_f32});
        defs.push_back({p + "ffn_gate_inp.bias", {experts}, tensor_f32});
        defs.push_back({p + "ffn_gate_exps.weight", {kDim, kDim, experts}, tensor_mxfp4});
        defs.push_back({p + "ffn_gate_exps.bias", {kDim, experts}, tensor_f32});
        defs.push_back({p + "ffn_up_exps.weight", {kDim, kDim, experts}, tensor_mxfp4});
        defs.push_back({p + "ffn_up_exps.bias", {kDim, experts}, tensor_f32});
        defs.push_back({p + "ffn_down_exps.weight", {kDim, kDim, experts}, tensor_mxfp4});
        defs.push_back({p + "ffn_down_exps.bias", {kDim, experts}, tensor_f32});
    }

    std::string meta;
    key_str(meta, "general.architecture", "gpt-oss");
    key_u32(meta, "gpt-oss.block_count", uint32_t(layers));
    key_u32(meta, "gpt-oss.context_length", 131072);
    key_u32(meta, "gpt-oss.embedding_length", kDim);
    key_u32(meta, "gpt-oss.feed_forward_length", kDim);
    key_u32(meta, "gpt-oss.attention.head_count", 64);
    key_u32(meta, "gpt-oss.attention.head_count_kv", 8);
    key_u32(meta, "gpt-oss.attention.key_length", 64);
    key_u32(meta, "gpt-oss.attention.value_length", 64);
    key_u32(meta, "gpt-oss.expert_used_count", 4);
    key_u32(meta, "gpt-oss.expert_feed_forward_length", kDim);
    key_u32(meta, "gpt-oss.attention.sliding_window", 128);
    key_f32(meta, "gpt-oss.attention.layer_norm_rms_epsilon", 1.0e-5f);
    key_f32(meta, "gpt-oss.rope.freq_base", 150000.0f);
    key_f32(meta, "gpt-oss.rope.scaling.factor", 32.0f);
    key_u32(meta, "gpt-oss.rope.scaling.original_context_length", 4096);
    key_f32(meta, "gpt-oss.rope.scaling.yarn_beta_fast", 32.0f);
    key_f32(meta, "gpt-oss.rope.scaling.yarn_beta_slow", 1.0f);
    key_u32(meta, "gpt-oss.expert_count", uint32_t(experts));
    const uint64_t key_count = 19;

    std::string file;
    put_u32(file, 0x46554747u); // "GGUF"
    put_u32(file, 3);
    put_u64(file, defs.size());
    put_u64(file, key_count);
    file += meta;
    uint64_t largest = 0;
    for (const TensorDef &t : defs) {
        put_str(file, t.name);
        put_u32(file, uint32_t(t.shape.size()));
        for (uint64_t d : t.shape) {
            put_u64(file, d);
        }
        put_u32(file, t.type);
        put_u64(file, 0);
        largest = std::max(largest, def_bytes(t));
    }
    file.append((32 - file.size() % 32) % 32, '\0');
    const uint64_t total = file.size() + largest;

    char path[] = "/tmp/ttl-ref-gguf-XXXXXX";
    const int fd = mkstemp(path);
    if (fd < 0) {
        throw std::runtime_error("cannot create reference fixture file");
    }
    bool ok = ::write(fd, file.data(), file.size()) == ssize_t(file.size());
    ok = ok && ftruncate(fd, off_t(total)) == 0;
    close(fd);
    if (!ok) {
        unlink(path);
        throw std::runtime_error("cannot write reference fixture file");
    }
    return path;
}

// One metadata file, GgufFile and GptOssModel per (experts, capacity).
struct RefModel {
    std::string path;
    std::unique_ptr<GgufFile> file;
    std::unique_ptr<GptOssModel> model;
    size_t experts = 0;
    size_t capacity = 0;

    ~RefModel() {
        model.reset();
        file.reset();
        if (!path.empty()) {
            unlink(path.c_str());
        }
    }
};

std::unordered_map<uint64_t, std::unique_ptr<RefModel>> g_models;

RefModel &get_model(size_t experts, size_t capacity) {
    const uint64_t key = (uint64_t(experts) << 32) | capacity;
    auto found = g_models.find(key);
    if (found != g_models.end()) {
        return *found->second;
    }
    auto m = std::make_unique<RefModel>();
    m->experts = experts;
    m->capacity = capacity;
    m->path = write_fixture(experts);
    m->file = std::make_unique<GgufFile>(m->path.c_str());
    m->model = std::make_unique<GptOssModel>(*m->file, capacity, std::string(), capacity);
    RefModel &ref = *m;
    g_models.emplace(key, std::move(m));
    return ref;
}

GgufTensor *find_tensor(GgufFile &file, std::string_view name) {
    auto &tensors = file.*member(TagTensors{});
    for (GgufTensor &t : tensors) {
        if (t.name == name) {
            return &t;
        }
    }
    throw std::runtime_error("fixture tensor missing: " + std::string(name));
}

struct LayerBuffers {
    const float *router_w, *router_b;
    const uint8_t *gate_w;
    const float *gate_b;
    const uint8_t *up_w;
    const float *up_b;
    const uint8_t *down_w;
    const float *down_b;
};

void bind_layer0(RefModel &m, const LayerBuffers &b) {
    GgufFile &f = *m.file;
    find_tensor(f, "blk.0.ffn_gate_inp.weight")->data = (const std::byte *)b.router_w;
    find_tensor(f, "blk.0.ffn_gate_inp.bias")->data = (const std::byte *)b.router_b;
    find_tensor(f, "blk.0.ffn_gate_exps.weight")->data = (const std::byte *)b.gate_w;
    find_tensor(f, "blk.0.ffn_gate_exps.bias")->data = (const std::byte *)b.gate_b;
    find_tensor(f, "blk.0.ffn_up_exps.weight")->data = (const std::byte *)b.up_w;
    find_tensor(f, "blk.0.ffn_up_exps.bias")->data = (const std::byte *)b.up_b;
    find_tensor(f, "blk.0.ffn_down_exps.weight")->data = (const std::byte *)b.down_w;
    find_tensor(f, "blk.0.ffn_down_exps.bias")->data = (const std::byte *)b.down_b;
}

template <class F> int guarded(F &&body) {
    try {
        body();
        return 0;
    } catch (const std::exception &e) {
        g_error = e.what();
        return -1;
    }
}

GgufTensor view(const void *data, std::vector<uint64_t> shape, uint32_t type) {
    GgufTensor t;
    t.name = "view";
    t.shape = std::move(shape);
    t.type = type;
    t.offset = 0;
    t.data = (const std::byte *)data;
    return t;
}

// A model of its own for one worker thread (GptOssModel keeps its scratch in
// members, so threads never share one): `layers` layers, room for one token.
std::unique_ptr<RefModel> make_model(size_t experts, size_t layers) {
    auto m = std::make_unique<RefModel>();
    m->experts = experts;
    m->capacity = 1;
    m->path = write_fixture(experts, layers);
    m->file = std::make_unique<GgufFile>(m->path.c_str());
    m->model = std::make_unique<GptOssModel>(*m->file, 1, std::string(), 1);
    return m;
}

// Aims layer l's MoE tensors at a caller's buffers: eight pointers in the
// order router_w, router_b, gate_w, gate_b, up_w, up_b, down_w, down_b.
void bind_layer(RefModel &m, size_t l, const void *const *p) {
    GgufFile &f = *m.file;
    const std::string b = "blk." + std::to_string(l) + ".";
    static const char *const names[8] = {"ffn_gate_inp.weight", "ffn_gate_inp.bias", "ffn_gate_exps.weight",
                                         "ffn_gate_exps.bias",  "ffn_up_exps.weight", "ffn_up_exps.bias",
                                         "ffn_down_exps.weight", "ffn_down_exps.bias"};
    for (int k = 0; k < 8; ++k) {
        find_tensor(f, b + names[k])->data = (const std::byte *)p[k];
    }
}

// One (token, layer) step of GptOssModel::forward without the attention block
// (src/model.cpp:590-594): normalized = rms_norm(x, norm), out = moe(layer l,
// normalized), y = x + out; the router logits stay in the model (router_).
void forward_step(GptOssModel &model, size_t l, const float *norm_w, const float *ones, const float *x, float *y,
                  float *normalized, float *out) {
    const GgufTensor g = view(norm_w ? norm_w : ones, {kDim}, tensor_f32);
    rms_norm(x, g, 1.0e-5f, normalized);
    auto &layers = model.*member(TagLayers{});
    (model.*member(TagMoe{}))(layers[l], normalized, out, l, 0);
    for (size_t j = 0; j < kDim; ++j) {
        y[j] = x[j] + out[j];
    }
}

// Runs body(worker, model) on `threads` threads, each with its own model;
// rethrows the first failure.
template <class F> void run_workers(size_t experts, size_t layers, int threads, F &&body) {
    const int n = std::max(1, threads);
    std::vector<std::unique_ptr<RefModel>> models;
    for (int i = 0; i < n; ++i) {
        models.push_back(make_model(experts, layers));
    }
    std::vector<std::string> errors(static_cast<size_t>(n));
    std::vector<std::thread> pool;
    for (int i = 0; i < n; ++i) {
        pool.emplace_back([&, i] {
            try {
                body(i, *models[size_t(i)]);
            } catch (const std::exception &e) {
                errors[size_t(i)] = e.what();
            }
        });
    }
    for (std::thread &t : pool) {
        t.join();
    }
    for (const std::string &e : errors) {
        if (!e.empty()) {
            throw std::runtime_error(e);
        }
    }
}

} // namespace

// Direct handles on the two ISA clones of the reference's multiversioned
// kernels (GCC names the v4 body with an ".arch_x86_64_v4" suffix), used the
// way tests/host_dispatch.cpp:16-21 does for its own kernels.
void matvec_v4(const GgufTensor &, const GgufTensor &, const float *, float *,
                            size_t) asm("_Z21matvec_add_mxfp4_2880RK10GgufTensorS1_PKfPfm.arch_x86_64_v4");
void matvec_default(const GgufTensor &, const GgufTensor &, const float *, float *,
                                 size_t) asm("_Z21matvec_add_mxfp4_2880RK10GgufTensorS1_PKfPfm");
void matmul_v4(const GgufTensor &, const GgufTensor &, const float *, const size_t *, size_t, float *,
                            float *, size_t)
    asm("_Z36matmul_add_mxfp4_selected_transposedRK10GgufTensorS1_PKfPKmmPfS6_m.arch_x86_64_v4");
void matmul_default(const GgufTensor &, const GgufTensor &, const float *, const size_t *, size_t,
                                 float *, float *, size_t)
    asm("_Z36matmul_add_mxfp4_selected_transposedRK10GgufTensorS1_PKfPKmmPfS6_m");


extern "C" {

// The attention block of GptOssModel::forward (src/model.cpp:578-590) for
// positions 0 .. positions-1 of layer `layer_index` (even: a sliding-window
// layer, odd: a full one), through tt-lab's own code: rms_norm,
// matvec_add_q8_0 for Q / K / V, the model's apply_rope, store_kv and
// attention_from_cache, matvec_add_q8_0 for the output, residual add.  The
// layer's attention tensors are aimed at the caller's ten buffers (attn_norm,
// q_w, q_b, k_w, k_b, v_w, v_b, o_w, o_b, sinks).  x and residual are
// [positions][2880]; attended (optional) [positions][4096].
int tref_attention_steps(const void *const *tensors, int layer_index, size_t positions, const float *x,
                         float *residual, float *attended) {
    return guarded([&] {
        if (layer_index < 0 || layer_index > 1 || positions == 0) {
            throw std::runtime_error("layer_index must be 0 or 1 and positions > 0");
        }
        const std::string path = write_fixture(32);
        GgufFile file(path.c_str());
        static const char *const names[10] = {"attn_norm.weight", "attn_q.weight",      "attn_q.bias",
                                              "attn_k.weight",    "attn_k.bias",        "attn_v.weight",
                                              "attn_v.bias",      "attn_output.weight", "attn_output.bias",
                                              "attn_sinks.weight"};
        const std::string b = "blk." + std::to_string(layer_index) + ".";
        for (int k = 0; k < 10; ++k) {
            find_tensor(file, b + names[k])->data = (const std::byte *)tensors[k];
        }
        GptOssModel model(file, positions, std::string(), 1);
        auto &layer = (model.*member(TagLayers{}))[size_t(layer_index)];
        std::vector<float> normalized(kDim), q(4096), k(512), v(512), att(4096), proj(kDim);
        for (size_t p = 0; p < positions; ++p) {
            const float *xp = x + p * kDim;
            rms_norm(xp, *layer.attention_norm, 1.0e-5f, normalized.data());
            matvec_add_q8_0(*layer.query_weight, *layer.query_bias, normalized.data(), q.data());
            matvec_add_q8_0(*layer.key_weight, *layer.key_bias, normalized.data(), k.data());
            matvec_add_q8_0(*layer.value_weight, *layer.value_bias, normalized.data(), v.data());
            (model.*member(TagRope{}))(q.data(), 64, p);
            (model.*member(TagRope{}))(k.data(), 8, p);
            (model.*member(TagStoreKv{}))(layer, p, k.data(), v.data());
            (model.*member(TagAttend{}))(layer, size_t(layer_index), p, q.data(), att.data());
            matvec_add_q8_0(*layer.attention_output_weight, *layer.attention_output_bias, att.data(), proj.data());
            for (size_t j = 0; j < kDim; ++j) {
                residual[p * kDim + j] = xp[j] + proj[j];
            }
            if (attended) {
                std::memcpy(attended + p * 4096, att.data(), 4096 * sizeof(float));
            }
        }
        unlink(path.c_str());
    });
}

const char *tref_last_error() {
    return g_error.c_str();
}

// 1 when the ifunc resolver picks the AVX-512 (x86-64-v4) clones on this host.
int tref_isa_v4() {
    return __builtin_cpu_supports("x86-64-v4") ? 1 : 0;
}

// The reference's MXFP4 matvec (src/tensor.cpp:239-304) on `experts` packed
// experts.  isa: -1 dispatched, 0 default clone, 1 v4 clone.
int tref_matvec_add_mxfp4(const uint8_t *w, const float *bias, size_t experts, size_t expert, const float *x,
                          float *y, int isa) {
    return guarded([&] {
        const GgufTensor m = view(w, {kDim, kDim, experts}, tensor_mxfp4);
        const GgufTensor b = view(bias, {kDim, experts}, tensor_f32);
        if (isa == 1) {
            if (!tref_isa_v4()) {
                throw std::runtime_error("host lacks x86-64-v4");
            }
            matvec_v4(m, b, x, y, expert);
        } else if (isa == 0) {
            matvec_default(m, b, x, y, expert);
        } else {
            matvec_add_mxfp4_2880(m, b, x, y, expert);
        }
    });
}

// The reference's selected-token matmul (src/tensor.cpp:319-495).
int tref_matmul_add_mxfp4_selected(const uint8_t *w, const float *bias, size_t experts, size_t expert,
                                   const float *xt, const size_t *tokens, size_t n, float *out, int isa) {
    return guarded([&] {
        const GgufTensor m = view(w, {kDim, kDim, experts}, tensor_mxfp4);
        const GgufTensor b = view(bias, {kDim, experts}, tensor_f32);
        std::vector<float> workspace(4 * n);
        if (isa == 1) {
            if (!tref_isa_v4()) {
                throw std::runtime_error("host lacks x86-64-v4");
            }
            matmul_v4(m, b, xt, tokens, n, out, workspace.data(), expert);
        } else if (isa == 0) {
            matmul_default(m, b, xt, tokens, n, out, workspace.data(), expert);
        } else {
            matmul_add_mxfp4_selected_transposed(m, b, xt, tokens, n, out, workspace.data(), expert);
        }
    });
}

float tref_mxfp4_scale(uint8_t e) {
    return mxfp4_scale(e);
}

int tref_rms_norm(const float *x, const float *g, float eps, float *out, size_t n) {
    return guarded([&] {
        const GgufTensor w = view(g, {n}, tensor_f32);
        rms_norm(x, w, eps, out);
    });
}

// GptOssModel::moe (src/model.cpp:292-338) on one token.
int tref_moe_decode(size_t experts, const float *router_w, const float *router_b, const uint8_t *gate_w,
                    const float *gate_b, const uint8_t *up_w, const float *up_b, const uint8_t *down_w,
                    const float *down_b, const float *x, float *out, int32_t *idx, float *w) {
    return guarded([&] {
        RefModel &m = get_model(experts, 1);
        bind_layer0(m, {router_w, router_b, gate_w, gate_b, up_w, up_b, down_w, down_b});
        GptOssModel &model = *m.model;
        auto &layers = model.*member(TagLayers{});
        (model.*member(TagMoe{}))(layers[0], x, out, 0, 0);
        const auto &indices = model.*member(TagIndices{});
        const auto &weights = model.*member(TagWeights{});
        for (size_t i = 0; i < 4; ++i) {
            if (idx) {
                idx[i] = int32_t(indices[i]);
            }
            if (w) {
                w[i] = weights[i];
            }
        }
    });
}

// GptOssModel::moe_batch (src/model.cpp:340-461) on `tokens` tokens.
int tref_moe_prefill(size_t experts, const float *router_w, const float *router_b, const uint8_t *gate_w,
                     const float *gate_b, const uint8_t *up_w, const float *up_b, const uint8_t *down_w,
                     const float *down_b, const float *x, size_t tokens, float *out, int32_t *idx, float *w) {
    return guarded([&] {
        // Capacities are rounded up so repeated calls reuse one model.
        size_t capacity = 64;
        while (capacity < tokens) {
            capacity *= 2;
        }
        RefModel &m = get_model(experts, capacity);
        bind_layer0(m, {router_w, router_b, gate_w, gate_b, up_w, up_b, down_w, down_b});
        GptOssModel &model = *m.model;
        auto &layers = model.*member(TagLayers{});
        (model.*member(TagMoeBatch{}))(layers[0], x, out, 0, tokens);
        const auto &indices = model.*member(TagIndicesSeq{});
        const auto &weights = model.*member(TagWeightsSeq{});
        for (size_t i = 0; i < tokens * 4; ++i) {
            if (idx) {
                idx[i] = int32_t(indices[i]);
            }
            if (w) {
                w[i] = weights[i];
            }
        }
    });
}

// Expert-parallel harness for the CPU baseline: the reference's router
// (matvec_add_f32) and per-expert MXFP4 kernels on host threads, combine kept
// serial in rank order as in src/model.cpp:323-337.  The selection and softmax
// are src/model.cpp:296-321 restated.  threads = 1: the reference's own
// single-threaded order; 2..4: one thread per selected expert (gate, up,
// down); 8: the eight gate and up products at once, each expert's down after
// its up (the most the unmodified whole-matrix kernels can overlap).
int tref_moe_decode_threaded(size_t experts, const float *router_w, const float *router_b, const uint8_t *gate_w,
                             const float *gate_b, const uint8_t *up_w, const float *up_b, const uint8_t *down_w,
                             const float *down_b, const float *x, float *out, int threads) {
    return guarded([&] {
        const GgufTensor rw = view(router_w, {kDim, experts}, tensor_f32);
        const GgufTensor rb = view(router_b, {experts}, tensor_f32);
        const GgufTensor gw = view(gate_w, {kDim, kDim, experts}, tensor_mxfp4);
        const GgufTensor gb = view(gate_b, {kDim, experts}, tensor_f32);
        const GgufTensor uw = view(up_w, {kDim, kDim, experts}, tensor_mxfp4);
        const GgufTensor ub = view(up_b, {kDim, experts}, tensor_f32);
        const GgufTensor dw = view(down_w, {kDim, kDim, experts}, tensor_mxfp4);
        const GgufTensor db = view(down_b, {kDim, experts}, tensor_f32);
        std::vector<float> router(experts);
        matvec_add_f32(rw, rb, x, router.data());
        std::vector<size_t> order(experts);
        for (size_t i = 0; i < experts; ++i) {
            order[i] = i;
        }
        for (size_t i = 0; i < 4; ++i) {
            size_t best = i;
            for (size_t j = i + 1; j < experts; ++j) {
                if (router[order[j]] > router[order[best]]) {
                    best = j;
                }
            }
            std::swap(order[i], order[best]);
        }
        float maximum = -std::numeric_limits<float>::infinity();
        for (size_t i = 0; i < 4; ++i) {
            maximum = std::max(maximum, router[order[i]]);
        }
        float weights[4];
        float sum = 0.0f;
        for (size_t i = 0; i < 4; ++i) {
            weights[i] = std::exp(router[order[i]] - maximum);
            sum += weights[i];
        }
        for (size_t i = 0; i < 4; ++i) {
            weights[i] /= sum;
        }
        std::vector<float> down(4 * kDim);
        auto run_expert = [&](size_t sel) {
            std::vector<float> gate(kDim), up(kDim), hidden(kDim);
            const size_t e = order[sel];
            matvec_add_mxfp4_2880(gw, gb, x, gate.data(), e);
            matvec_add_mxfp4_2880(uw, ub, x, up.data(), e);
            for (size_t i = 0; i < kDim; ++i) {
                const float a = std::min(gate[i], 7.0f);
                const float b = std::clamp(up[i], -7.0f, 7.0f);
                hidden[i] = (a / (1.0f + std::exp(-1.702f * a))) * (b + 1.0f);
            }
            matvec_add_mxfp4_2880(dw, db, hidden.data(), down.data() + sel * kDim, e);
        };
        const size_t n = size_t(std::clamp(threads, 1, 8));
        if (n == 1) {
            for (size_t sel = 0; sel < 4; ++sel) {
                run_expert(sel);
            }
        } else if (n >= 8) {
            // threads 0-3: gate of expert t, then (once thread t + 4 has its
            // up) SwiGLU and down; threads 4-7: up of expert t - 4
            std::vector<float> gate(4 * kDim), up(4 * kDim);
            std::array<std::unique_ptr<std::latch>, 4> up_done;
            for (auto &l : up_done) {
                l = std::make_unique<std::latch>(1);
            }
            std::vector<std::thread> pool;
            for (size_t t = 0; t < 8; ++t) {
                pool.emplace_back([&, t] {
                    const size_t sel = t & 3;
                    const size_t e = order[sel];
                    if (t >= 4) {
                        matvec_add_mxfp4_2880(uw, ub, x, up.data() + sel * kDim, e);
                        up_done[sel]->count_down();
                        return;
                    }
                    matvec_add_mxfp4_2880(gw, gb, x, gate.data() + sel * kDim, e);
                    up_done[sel]->wait();
                    std::vector<float> hidden(kDim);
                    for (size_t i = 0; i < kDim; ++i) {
                        const float a = std::min(gate[sel * kDim + i], 7.0f);
                        const float b = std::clamp(up[sel * kDim + i], -7.0f, 7.0f);
                        hidden[i] = (a / (1.0f + std::exp(-1.702f * a))) * (b + 1.0f);
                    }
                    matvec_add_mxfp4_2880(dw, db, hidden.data(), down.data() + sel * kDim, e);
                });
            }
            for (std::thread &th : pool) {
                th.join();
            }
        } else {
            std::vector<std::thread> pool;
            for (size_t t = 0; t < n; ++t) {
                pool.emplace_back([&, t] {
                    for (size_t sel = t; sel < 4; sel += n) {
                        run_expert(sel);
                    }
                });
            }
            for (std::thread &th : pool) {
                th.join();
            }
        }
        std::fill(out, out + kDim, 0.0f);
        for (size_t sel = 0; sel < 4; ++sel) {
            for (size_t i = 0; i < kDim; ++i) {
                out[i] += weights[sel] * down[sel * kDim + i];
            }
        }
    });
}

// One layer for many tokens (the parity tests' checker): for each token t,
// y[t] = x[t] + moe(rms_norm(x[t], norm_w)) with tt-lab's own rms_norm and
// GptOssModel::moe, on `threads` host threads (each token's arithmetic is the
// single-threaded reference's).  layer: the eight tensor pointers of
// bind_layer; norm_w NULL = ones.  idx/w [T][4] and logits [T][E] optional.
int tref_moe_layer_tokens(size_t experts, const void *const *layer, const float *norm_w, const float *x, float *y,
                          size_t tokens, int threads, int32_t *idx, float *w, float *logits) {
    return guarded([&] {
        const std::vector<float> ones(kDim, 1.0f);
        std::atomic<size_t> next{0};
        run_workers(experts, 24, int(std::min<size_t>(size_t(std::max(threads, 1)), std::max<size_t>(tokens, 1))),
                    [&](int, RefModel &m) {
                        bind_layer(m, 0, layer);
                        GptOssModel &model = *m.model;
                        std::vector<float> normalized(kDim), out(kDim);
                        for (size_t t = next++; t < tokens; t = next++) {
                            forward_step(model, 0, norm_w, ones.data(), x + t * kDim, y + t * kDim,
                                         normalized.data(), out.data());
                            const auto &indices = model.*member(TagIndices{});
                            const auto &weights = model.*member(TagWeights{});
                            const auto &router = model.*member(TagRouter{});
                            for (size_t i = 0; i < 4; ++i) {
                                if (idx) {
                                    idx[t * 4 + i] = int32_t(indices[i]);
                                }
                                if (w) {
                                    w[t * 4 + i] = weights[i];
                                }
                            }
                            if (logits) {
                                std::copy(router.begin(), router.begin() + experts, logits + t * experts);
                            }
                        }
                    });
    });
}

// Token-major decode of independent tokens, as GptOssModel::forward runs one
// token through every layer (src/model.cpp:574-597, attention left out): each
// of `threads` workers takes the next token and runs it through layers
// [0, layers).  tables: 8 tensor pointers per layer (bind_layer's order);
// norms: one RMSNorm weight pointer per layer (NULL entries or a NULL array =
// ones).  y may alias x.
int tref_forward_tokens(size_t experts, size_t layers, const void *const *tables, const float *const *norms,
                        const float *x, float *y, size_t tokens, int threads) {
    return guarded([&] {
        if (layers == 0 || layers > 36) {
            throw std::runtime_error("layers must be in 1..36");
        }
        const std::vector<float> ones(kDim, 1.0f);
        std::atomic<size_t> next{0};
        const size_t fixture_layers = layers > 24 ? 36 : 24;
        run_workers(experts, fixture_layers,
                    int(std::min<size_t>(size_t(std::max(threads, 1)), std::max<size_t>(tokens, 1))),
                    [&](int, RefModel &m) {
                        for (size_t l = 0; l < layers; ++l) {
                            bind_layer(m, l, tables + 8 * l);
                        }
                        GptOssModel &model = *m.model;
                        std::vector<float> cur(kDim), nxt(kDim), normalized(kDim), out(kDim);
                        for (size_t t = next++; t < tokens; t = next++) {
                            std::copy(x + t * kDim, x + (t + 1) * kDim, cur.begin());
                            for (size_t l = 0; l < layers; ++l) {
                                forward_step(model, l, norms ? norms[l] : nullptr, ones.data(), cur.data(),
                                             nxt.data(), normalized.data(), out.data());
                                cur.swap(nxt);
                            }
                            std::copy(cur.begin(), cur.end(), y + t * kDim);
                        }
                    });
    });
}

// tt-lab's output head on caller buffers: matvec_q8_0 (src/tensor.cpp:202-218)
// over `rows` rows of a Q8_0 matrix, then, when rows is the model's vocabulary,
// GptOssModel::greedy (src/model.cpp:604-612) on the result.
int tref_matvec_q8_0(const uint8_t *w, size_t rows, const float *x, float *y, int32_t *token) {
    return guarded([&] {
        const GgufTensor m = view(w, {kDim, rows}, tensor_q8_0);
        matvec_q8_0(m, x, y);
        if (token) {
            if (rows != 201088) {
                throw std::runtime_error("greedy needs the full vocabulary (201088 rows)");
            }
            *token = get_model(32, 1).model->greedy(y);
        }
    });
}

// GptOssModel::greedy (src/model.cpp:604-612) on a caller's full-vocabulary
// logit vector (201088 floats).
int tref_greedy(const float *logits, int32_t *token) {
    return guarded([&] { *token = get_model(32, 1).model->greedy(logits); });
}

} // extern "C"
