// cuda_check.cpp -- tt-lab's own GptOssModel::prefill / forward with the MoE
// on the GPU backend, checked against the same model on the CPU.
//
// TEST INFRASTRUCTURE ONLY: the compiled counterpart of the binding that the
// integration notes describe.  Built by oracle/Makefile (target `check`) into
// oracle/_ref/ttlab_cuda_check, linked against tt-lab's src/{tensor,gguf,
// model}.cpp compiled unmodified (oracle/_ref/libttlref.so) and the product
// library (libttl_moe.so).
//
// The hook: tt-lab's forward/prefill call the private members
// GptOssModel::moe / moe_batch (src/model.cpp:536, :591) through the shared
// library's symbol table (it is built with -fPIC and default visibility, so
// the calls are interposable).  This executable defines both members; the
// dynamic linker binds tt-lab's calls to these definitions, which route to
// ttl_moe_decode / ttl_moe_prefill when the model instance has the backend
// enabled and to the library's own definitions (dlsym(RTLD_NEXT)) otherwise.
// No tt-lab source is edited.
//
// The check mirrors run_device_proxy_check (src/tt_backend.cpp:3647-3714):
// two models over the same weights, one on the CPU and one with the MoE on
// the GPU, run the same prompt (prefill) and then greedy generation
// (forward), and the report gives, per token, the residual stream's rel-RMS
// and cosine (compare_vectors, src/tt_backend.cpp:3100-3128), per layer the
// MoE output's rel-RMS / cosine and the top-4 overlap and top-1 match, and the
// final logits' agreement and greedy token.  The weights are seeded
// synthetic tensors (no gpt-oss GGUF is available): a metadata-only GGUF
// fixture whose tensor views are pointed at host buffers.
#include <dlfcn.h>
#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf.h"
#include "model.h"
#include "tensor.h"
#include "ttl_moe.h"

extern "C" {
void oref_synth_normal(float *dst, size_t n, uint64_t seed, uint64_t stream, float sigma, float mean);
void oref_synth_mxfp4(uint8_t *dst, size_t blocks, uint64_t seed, uint64_t stream, uint32_t lo, uint32_t count);
void oref_synth_q8_0_range(uint8_t *dst, size_t b0, size_t blocks, uint64_t seed, uint64_t stream);
}

namespace {

// Private members reached with the explicit-instantiation access idiom.
template <class Tag, auto Member> struct Expose {
    friend auto member(Tag) {
        return Member;
    }
};
struct TagIdx {
    friend auto member(TagIdx);
};
struct TagIdxSeq {
    friend auto member(TagIdxSeq);
};
struct TagTensors {
    friend auto member(TagTensors);
};

} // namespace

template struct Expose<TagIdx, &GptOssModel::expert_indices_>;
template struct Expose<TagIdxSeq, &GptOssModel::expert_indices_sequence_>;
template struct Expose<TagTensors, &GgufFile::tensors_>;

namespace {

constexpr size_t kDim = 2880;
constexpr size_t kVocab = 201088;
constexpr size_t kLayers = 24;
constexpr size_t kExperts = 32;

// ---- per-model hook state ----
struct Trace {
    std::vector<std::vector<float>> moe_out;     // [call] 2880 x count
    std::vector<std::vector<int32_t>> top4;      // [call] 4 x count
};
struct Hook {
    ttl_moe *gpu = nullptr;  // null: the CPU path
    Trace trace;
    size_t calls = 0;
};
std::map<const GptOssModel *, Hook> g_hooks;

template <class T> T next_symbol(const char *name) {
    void *p = dlsym(RTLD_NEXT, name);
    if (!p) {
        throw std::runtime_error(std::string("tt-lab symbol not found: ") + name);
    }
    T fn;
    std::memcpy(&fn, &p, sizeof(p));
    return fn;
}

void check(int rc, const char *what) {
    if (rc != TTL_OK) {
        throw std::runtime_error(std::string(what) + ": " + ttl_moe_last_error(nullptr));
    }
}

} // namespace

// ---- the interposed members ----
using CpuMoe = void (*)(GptOssModel *, const void *, const float *, float *, size_t, size_t);

void GptOssModel::moe(const Layer &layer, const float *input, float *output, size_t layer_index, size_t position) {
    static const CpuMoe cpu = next_symbol<CpuMoe>("_ZN11GptOssModel3moeERKNS_5LayerEPKfPfmm");
    Hook &h = g_hooks[this];
    ++h.calls;
    std::vector<int32_t> idx(4);
    if (h.gpu) {
        float w[4];
        if (ttl_moe_decode(h.gpu, int(layer_index), input, output, idx.data(), w) != TTL_OK) {
            throw std::runtime_error(std::string("cuda moe: ") + ttl_moe_last_error(h.gpu));
        }
    } else {
        cpu(this, &layer, input, output, layer_index, position);
        const auto &ei = this->*member(TagIdx{});
        for (int k = 0; k < 4; ++k) {
            idx[size_t(k)] = int32_t(ei[size_t(k)]);
        }
    }
    h.trace.moe_out.emplace_back(output, output + kDim);
    h.trace.top4.push_back(idx);
}

void GptOssModel::moe_batch(const Layer &layer, const float *input, float *output, size_t layer_index,
                            size_t count) {
    static const CpuMoe cpu = next_symbol<CpuMoe>("_ZN11GptOssModel9moe_batchERKNS_5LayerEPKfPfmm");
    Hook &h = g_hooks[this];
    ++h.calls;
    std::vector<int32_t> idx(4 * count);
    if (h.gpu) {
        std::vector<float> w(4 * count);
        if (ttl_moe_prefill(h.gpu, int(layer_index), input, count, output, idx.data(), w.data()) != TTL_OK) {
            throw std::runtime_error(std::string("cuda moe_batch: ") + ttl_moe_last_error(h.gpu));
        }
    } else {
        cpu(this, &layer, input, output, layer_index, count);
        const auto &seq = this->*member(TagIdxSeq{});
        for (size_t i = 0; i < 4 * count; ++i) {
            idx[i] = int32_t(seq[i]);
        }
    }
    h.trace.moe_out.emplace_back(output, output + kDim * count);
    h.trace.top4.push_back(idx);
}

namespace {

// ---- a metadata-only gpt-oss GGUF whose tensors all sit at offset 0 ----
void put(std::string &o, const void *p, size_t n) {
    o.append(static_cast<const char *>(p), n);
}
void put_u32(std::string &o, uint32_t v) {
    put(o, &v, 4);
}
void put_u64(std::string &o, uint64_t v) {
    put(o, &v, 8);
}
void put_str(std::string &o, const std::string &s) {
    put_u64(o, s.size());
    o += s;
}
void key_u32(std::string &o, const char *k, uint32_t v) {
    put_str(o, k);
    put_u32(o, 4);
    put_u32(o, v);
}
void key_f32(std::string &o, const char *k, float v) {
    put_str(o, k);
    put_u32(o, 6);
    put(o, &v, 4);
}

struct Def {
    std::string name;
    std::vector<uint64_t> shape;
    uint32_t type;
};

uint64_t def_bytes(const Def &d) {
    uint64_t n = 1;
    for (uint64_t s : d.shape) {
        n *= s;
    }
    return d.type == tensor_f32 ? 4 * n : d.type == tensor_q8_0 ? n / 32 * 34 : n / 32 * 17;
}

std::vector<Def> model_defs() {
    std::vector<Def> d;
    d.push_back({"token_embd.weight", {kDim, kVocab}, tensor_q8_0});
    d.push_back({"output_norm.weight", {kDim}, tensor_f32});
    d.push_back({"output.weight", {kDim, kVocab}, tensor_q8_0});
    for (size_t i = 0; i < kLayers; ++i) {
        const std::string p = "blk." + std::to_string(i) + ".";
        d.push_back({p + "attn_norm.weight", {kDim}, tensor_f32});
        d.push_back({p + "post_attention_norm.weight", {kDim}, tensor_f32});
        d.push_back({p + "attn_q.weight", {kDim, 4096}, tensor_q8_0});
        d.push_back({p + "attn_q.bias", {4096}, tensor_f32});
        d.push_back({p + "attn_k.weight", {kDim, 512}, tensor_q8_0});
        d.push_back({p + "attn_k.bias", {512}, tensor_f32});
        d.push_back({p + "attn_v.weight", {kDim, 512}, tensor_q8_0});
        d.push_back({p + "attn_v.bias", {512}, tensor_f32});
        d.push_back({p + "attn_output.weight", {4096, kDim}, tensor_q8_0});
        d.push_back({p + "attn_output.bias", {kDim}, tensor_f32});
        d.push_back({p + "attn_sinks.weight", {64}, tensor_f32});
        d.push_back({p + "ffn_gate_inp.weight", {kDim, kExperts}, tensor_f32});
        d.push_back({p + "ffn_gate_inp.bias", {kExperts}, tensor_f32});
        d.push_back({p + "ffn_gate_exps.weight", {kDim, kDim, kExperts}, tensor_mxfp4});
        d.push_back({p + "ffn_gate_exps.bias", {kDim, kExperts}, tensor_f32});
        d.push_back({p + "ffn_up_exps.weight", {kDim, kDim, kExperts}, tensor_mxfp4});
        d.push_back({p + "ffn_up_exps.bias", {kDim, kExperts}, tensor_f32});
        d.push_back({p + "ffn_down_exps.weight", {kDim, kDim, kExperts}, tensor_mxfp4});
        d.push_back({p + "ffn_down_exps.bias", {kDim, kExperts}, tensor_f32});
    }
    return d;
}

std::string write_fixture(const std::vector<Def> &defs) {
    std::string meta;
    put_str(meta, "general.architecture");
    put_u32(meta, 8);
    put_str(meta, "gpt-oss");
    key_u32(meta, "gpt-oss.block_count", uint32_t(kLayers));
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
    key_u32(meta, "gpt-oss.expert_count", uint32_t(kExperts));
    std::string f;
    put_u32(f, 0x46554747u);
    put_u32(f, 3);
    put_u64(f, defs.size());
    put_u64(f, 19);
    f += meta;
    uint64_t largest = 0;
    for (const Def &d : defs) {
        put_str(f, d.name);
        put_u32(f, uint32_t(d.shape.size()));
        for (uint64_t s : d.shape) {
            put_u64(f, s);
        }
        put_u32(f, d.type);
        put_u64(f, 0);
        largest = std::max(largest, def_bytes(d));
    }
    f.append((32 - f.size() % 32) % 32, '\0');
    char path[] = "/tmp/ttl-cuda-check-XXXXXX";
    const int fd = mkstemp(path);
    if (fd < 0) {
        throw std::runtime_error("cannot create the fixture file");
    }
    const bool ok = ::write(fd, f.data(), f.size()) == ssize_t(f.size()) &&
                    ftruncate(fd, off_t(f.size() + largest)) == 0;
    close(fd);
    if (!ok) {
        unlink(path);
        throw std::runtime_error("cannot write the fixture file");
    }
    return path;
}

// ---- seeded synthetic weights ----
constexpr uint64_t kSeed = 21;

std::vector<float> normal(size_t n, uint64_t stream, float sigma, float mean = 0.0f) {
    std::vector<float> v(n);
    oref_synth_normal(v.data(), n, kSeed, stream, sigma, mean);
    return v;
}
// Q8_0 rows; `shift` lowers every block's half scale by 2^shift (the
// generator's scales, 2^-11..2^-9, suit the output matrix; the attention
// projections take /4, which keeps the attention scores of the synthetic
// model in the usual single-digit range).
std::vector<uint8_t> q8(size_t rows, size_t cols, uint64_t stream, int shift = 0) {
    std::vector<uint8_t> v(rows * cols / 32 * 34);
    oref_synth_q8_0_range(v.data(), 0, rows * cols / 32, kSeed, stream);
    for (size_t b = 0; shift && b < v.size() / 34; ++b) {
        uint16_t h = uint16_t(v[34 * b] | (v[34 * b + 1] << 8));
        h = uint16_t(h - (shift << 10));
        v[34 * b] = uint8_t(h);
        v[34 * b + 1] = uint8_t(h >> 8);
    }
    return v;
}
std::vector<uint8_t> mx(uint64_t stream) {
    std::vector<uint8_t> v(kExperts * kDim * kDim / 32 * 17);
    oref_synth_mxfp4(v.data(), v.size() / 17, kSeed, stream, 119, 7);
    return v;
}

struct Weights {
    std::vector<uint8_t> embd, out;
    std::vector<float> out_norm;
    // attention and MoE tensors, two sets alternating over the layers
    struct Layer {
        std::vector<float> attn_norm, post_norm, qb, kb, vb, ob, sinks, rw, rb, gb, ub, db;
        std::vector<uint8_t> q, k, v, o, g, u, d;
    } layer[2];
};

Weights make_weights() {
    Weights w;
    w.embd = q8(kVocab, kDim, 1000);
    w.out = q8(kVocab, kDim, 1001);
    w.out_norm = normal(kDim, 1002, 0.02f, 1.0f);
    for (int s = 0; s < 2; ++s) {
        Weights::Layer &L = w.layer[s];
        const uint64_t b = 2000 + 100 * uint64_t(s);
        L.attn_norm = normal(kDim, b + 0, 0.02f, 1.0f);
        L.post_norm = normal(kDim, b + 1, 0.02f, 1.0f);
        L.q = q8(4096, kDim, b + 2, 2);
        L.qb = normal(4096, b + 3, 0.02f);
        L.k = q8(512, kDim, b + 4, 2);
        L.kb = normal(512, b + 5, 0.02f);
        L.v = q8(512, kDim, b + 6, 2);
        L.vb = normal(512, b + 7, 0.02f);
        L.o = q8(kDim, 4096, b + 8, 2);
        L.ob = normal(kDim, b + 9, 0.02f);
        L.sinks = normal(64, b + 10, 0.5f);
        L.rw = normal(kExperts * kDim, b + 11, 0.02f);
        L.rb = normal(kExperts, b + 12, 0.02f);
        L.g = mx(b + 13);
        L.gb = normal(kExperts * kDim, b + 14, 0.02f);
        L.u = mx(b + 15);
        L.ub = normal(kExperts * kDim, b + 16, 0.02f);
        L.d = mx(b + 17);
        L.db = normal(kExperts * kDim, b + 18, 0.02f);
    }
    return w;
}

void bind(GgufFile &f, const Weights &w) {
    auto &tensors = f.*member(TagTensors{});
    auto at = [&](const std::string &name, const void *p) {
        for (GgufTensor &t : tensors) {
            if (t.name == name) {
                t.data = static_cast<const std::byte *>(p);
                return;
            }
        }
        throw std::runtime_error("fixture tensor missing: " + name);
    };
    at("token_embd.weight", w.embd.data());
    at("output.weight", w.out.data());
    at("output_norm.weight", w.out_norm.data());
    for (size_t i = 0; i < kLayers; ++i) {
        const Weights::Layer &L = w.layer[i & 1];
        const std::string p = "blk." + std::to_string(i) + ".";
        at(p + "attn_norm.weight", L.attn_norm.data());
        at(p + "post_attention_norm.weight", L.post_norm.data());
        at(p + "attn_q.weight", L.q.data());
        at(p + "attn_q.bias", L.qb.data());
        at(p + "attn_k.weight", L.k.data());
        at(p + "attn_k.bias", L.kb.data());
        at(p + "attn_v.weight", L.v.data());
        at(p + "attn_v.bias", L.vb.data());
        at(p + "attn_output.weight", L.o.data());
        at(p + "attn_output.bias", L.ob.data());
        at(p + "attn_sinks.weight", L.sinks.data());
        at(p + "ffn_gate_inp.weight", L.rw.data());
        at(p + "ffn_gate_inp.bias", L.rb.data());
        at(p + "ffn_gate_exps.weight", L.g.data());
        at(p + "ffn_gate_exps.bias", L.gb.data());
        at(p + "ffn_up_exps.weight", L.u.data());
        at(p + "ffn_up_exps.bias", L.ub.data());
        at(p + "ffn_down_exps.weight", L.d.data());
        at(p + "ffn_down_exps.bias", L.db.data());
    }
}

// compare_vectors (src/tt_backend.cpp:3100-3128)
struct Metrics {
    double rel_rms = 0.0, cosine = 1.0, max_abs = 0.0;
};
Metrics compare(const float *a, const float *b, size_t n) {
    double aa = 0, bb = 0, ee = 0, ab = 0, mx = 0;
    for (size_t i = 0; i < n; ++i) {
        const double x = a[i], y = b[i];
        aa += x * x;
        bb += y * y;
        ee += (x - y) * (x - y);
        ab += x * y;
        mx = std::max(mx, std::fabs(x - y));
    }
    Metrics m;
    m.rel_rms = std::sqrt(ee / double(n)) / std::max(1e-30, std::sqrt(bb / double(n)));
    m.cosine = ab / std::sqrt(std::max(1e-30, aa * bb));
    m.max_abs = mx;
    return m;
}

} // namespace

int main(int argc, char **argv) {
    try {
        const size_t prompt = argc > 1 ? size_t(std::atoi(argv[1])) : 8;
        const size_t generate = argc > 2 ? size_t(std::atoi(argv[2])) : 4;
        const int device = argc > 3 ? std::atoi(argv[3]) : 0;
        const size_t capacity = prompt + generate + 1;

        const Weights w = make_weights();
        const std::vector<Def> defs = model_defs();
        const std::string path = write_fixture(defs);
        GgufFile cpu_file(path.c_str()), gpu_file(path.c_str());
        unlink(path.c_str());
        bind(cpu_file, w);
        bind(gpu_file, w);
        GptOssModel cpu(cpu_file, capacity, std::string(), capacity);
        GptOssModel gpu(gpu_file, capacity, std::string(), capacity);

        // the backend (the integration notes' enable_cuda): every layer's MoE
        // tensors from the model's own weights, the same host buffers
        ttl_moe_config cfg{};
        cfg.experts = kExperts;
        cfg.layers = kLayers;
        cfg.max_tokens = uint32_t(capacity);
        cfg.device = device;
        cfg.world = 1;
        ttl_moe *h = nullptr;
        check(ttl_moe_create(&cfg, &h), "ttl_moe_create");
        for (size_t i = 0; i < kLayers; ++i) {
            const Weights::Layer &L = w.layer[i & 1];
            if (ttl_moe_upload_layer(h, int(i), L.rw.data(), L.rb.data(), L.g.data(), L.gb.data(), L.u.data(),
                                     L.ub.data(), L.d.data(), L.db.data()) != TTL_OK) {
                throw std::runtime_error(std::string("upload: ") + ttl_moe_last_error(h));
            }
        }
        g_hooks[&gpu].gpu = h;
        g_hooks[&cpu].gpu = nullptr;

        // a seeded prompt, then greedy generation on each model's own logits
        std::vector<int32_t> tokens(prompt);
        {
            std::vector<float> r = normal(prompt, 3000, 1.0f);
            for (size_t i = 0; i < prompt; ++i) {
                tokens[i] = int32_t(uint32_t(std::fabs(r[i]) * 1e6f) % kVocab);
            }
        }
        const float *lc = cpu.prefill(tokens.data(), prompt);
        std::vector<float> logits_cpu(lc, lc + kVocab);
        const float *lg = gpu.prefill(tokens.data(), prompt);
        std::vector<float> logits_gpu(lg, lg + kVocab);
        std::vector<Metrics> logit_m{compare(logits_gpu.data(), logits_cpu.data(), kVocab)};
        std::vector<int> top_match{cpu.greedy(logits_cpu.data()) == gpu.greedy(logits_gpu.data())};
        int32_t next = cpu.greedy(logits_cpu.data());
        for (size_t t = 0; t < generate; ++t) {
            // both models take the CPU's token, as the proxy check feeds one sequence
            lc = cpu.forward(next, prompt + t);
            logits_cpu.assign(lc, lc + kVocab);
            lg = gpu.forward(next, prompt + t);
            logits_gpu.assign(lg, lg + kVocab);
            logit_m.push_back(compare(logits_gpu.data(), logits_cpu.data(), kVocab));
            top_match.push_back(cpu.greedy(logits_cpu.data()) == gpu.greedy(logits_gpu.data()));
            next = cpu.greedy(logits_cpu.data());
        }

        // per layer call: the MoE output (prefill: every token of the batch)
        // and the expert selection
        const Trace &tc = g_hooks[&cpu].trace;
        const Trace &tg = g_hooks[&gpu].trace;
        if (tc.moe_out.size() != tg.moe_out.size() || tc.moe_out.size() != kLayers * (1 + generate)) {
            throw std::runtime_error("the hook saw " + std::to_string(tg.moe_out.size()) + " GPU and " +
                                     std::to_string(tc.moe_out.size()) + " CPU MoE calls");
        }
        double moe_rel_sum = 0, moe_cos_min = 1;
        size_t overlap = 0, top1 = 0, selections = 0, close = 0, same4 = 0;
        for (size_t c = 0; c < tc.moe_out.size(); ++c) {
            const size_t n = tc.moe_out[c].size() / kDim;
            for (size_t k = 0; k < n; ++k) {
                const Metrics m = compare(tg.moe_out[c].data() + k * kDim, tc.moe_out[c].data() + k * kDim, kDim);
                moe_rel_sum += m.rel_rms;
                moe_cos_min = std::min(moe_cos_min, m.cosine);
                close += (m.cosine >= 0.9999) ? 1 : 0;
                const int32_t *a = tg.top4[c].data() + 4 * k;
                const int32_t *b = tc.top4[c].data() + 4 * k;
                for (int i = 0; i < 4; ++i) {
                    overlap += size_t(std::count(b, b + 4, a[i]));
                }
                top1 += (a[0] == b[0]) ? 1 : 0;
                same4 += std::equal(a, a + 4, b) ? 1 : 0;
                ++selections;
            }
        }
        double logit_rel_max = 0, logit_cos_min = 1;
        for (const Metrics &m : logit_m) {
            logit_rel_max = std::max(logit_rel_max, m.rel_rms);
            logit_cos_min = std::min(logit_cos_min, m.cosine);
        }
        const size_t tops = size_t(std::count(top_match.begin(), top_match.end(), 1));
        std::printf("cuda check: %zu prompt tokens (prefill through moe_batch) + %zu generated (forward through moe), "
                    "%zu layers\n",
                    prompt, generate, kLayers);
        std::printf("MoE: %zu token-layer selections, avg rel RMS %.6g, min cosine %.9f\n", selections,
                    moe_rel_sum / double(selections), moe_cos_min);
        std::printf("expert selection summary: avg top-4 overlap %.3f/4, top-1 match %.3f\n",
                    double(overlap) / double(selections), double(top1) / double(selections));
        std::printf("logits: max rel RMS %.6g, min cosine %.9f, greedy token matches %zu/%zu\n", logit_rel_max,
                    logit_cos_min, tops, top_match.size());
        std::printf("MoE outputs within cosine 0.9999 of the CPU's: %zu/%zu; identical ordered top-4: %zu/%zu\n", close,
                    selections, same4, selections);
        std::printf("{\"selections\": %zu, \"moe_close\": %zu, \"top4_identical\": %zu, "
                    "\"moe_rel_rms_avg\": %.9g, \"moe_cosine_min\": %.12f, "
                    "\"top4_overlap_avg\": %.6f, \"top1_match\": %.6f, \"logits_rel_rms_max\": %.9g, "
                    "\"logits_cosine_min\": %.12f, \"greedy_matches\": %zu, \"greedy_total\": %zu, "
                    "\"gpu_moe_calls\": %zu}\n",
                    selections, close, same4, moe_rel_sum / double(selections), moe_cos_min,
                    double(overlap) / double(selections),
                    double(top1) / double(selections), logit_rel_max, logit_cos_min, tops, top_match.size(),
                    g_hooks[&gpu].calls);
        ttl_moe_destroy(h);
        return 0;
    } catch (const std::exception &e) {
        std::fprintf(stderr, "error: %s\n", e.what());
        return 1;
    }
}
