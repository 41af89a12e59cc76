// requant.cpp -- `requant --cuda`: a gpt-oss GGUF to a TTQ file whose MoE
// expert matrices are in the GPU layout, and the packed-input upload that
// consumes it.
//
// tt-lab's write_requant (src/requant.cpp:415-504) turns every MXFP4 expert
// tensor into Tensix BFP8 strips (format 5) and the other tensors into bf16
// layouts (formats 1, 2).  For the CUDA backend the expert matrices become
// TTL_TTQ_FORMAT_MXFP4_GPU (6) records, produced by the GPU packer (lossless);
// the router weights and every f32 bias are kept exactly as stored
// (TTL_TTQ_FORMAT_F32 = 7), since the router's f32 chain decides the expert
// selection.  The container is tt-lab's (header and records of
// src/requant.h:31-52, written by ttq.cpp), so tt-lab's TtqFile
// (src/tt_backend.cpp:315-445) reads the result.
//
// The GGUF reader here is the file format's own definition (GGUF v3: header,
// metadata key/values, tensor directory, aligned data), mapped read-only;
// only the metadata keys and tensors the MoE path needs are looked at.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include <cuda_runtime.h>

#include "../csrc/internal.h"
#include "ttl_moe.h"

namespace {

constexpr uint32_t kGgufF32 = 0;
constexpr uint32_t kGgufMxfp4 = 39;  // src/tensor.h:13
constexpr uint64_t kDim = 2880;

struct GgufTensorView {
    uint32_t type = 0;
    std::vector<uint64_t> shape;
    const uint8_t *data = nullptr;
    uint64_t bytes = 0;
};

// A read-only mapping of a GGUF file: integer / string metadata and the
// tensor directory.
class GgufMap {
  public:
    explicit GgufMap(const char *path) {
        fd_ = ::open(path, O_RDONLY);
        if (fd_ < 0) {
            throw std::string("cannot open GGUF ") + path + ": " + std::strerror(errno);
        }
        struct stat st {};
        if (fstat(fd_, &st) != 0 || st.st_size < 24) {
            throw std::string("cannot stat GGUF ") + path;
        }
        size_ = size_t(st.st_size);
        void *m = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd_, 0);
        if (m == MAP_FAILED) {
            throw std::string("cannot mmap GGUF ") + path;
        }
        base_ = static_cast<const uint8_t *>(m);
        parse();
    }
    ~GgufMap() {
        if (base_) {
            munmap(const_cast<uint8_t *>(base_), size_);
        }
        if (fd_ >= 0) {
            ::close(fd_);
        }
    }
    GgufMap(const GgufMap &) = delete;
    GgufMap &operator=(const GgufMap &) = delete;

    uint64_t integer(const std::string &key) const {
        const auto it = ints_.find(key);
        if (it == ints_.end()) {
            throw std::string("GGUF metadata key missing: ") + key;
        }
        return it->second;
    }
    const std::string &string(const std::string &key) const {
        const auto it = strings_.find(key);
        if (it == strings_.end()) {
            throw std::string("GGUF metadata key missing: ") + key;
        }
        return it->second;
    }
    const GgufTensorView &tensor(const std::string &name) const {
        const auto it = tensors_.find(name);
        if (it == tensors_.end()) {
            throw std::string("GGUF tensor missing: ") + name;
        }
        return it->second;
    }

  private:
    template <class T> T take() {
        need(sizeof(T));
        T v;
        std::memcpy(&v, base_ + pos_, sizeof(T));
        pos_ += sizeof(T);
        return v;
    }
    void need(uint64_t n) const {
        if (pos_ > size_ || n > size_ - pos_) {
            throw std::string("GGUF file is truncated");
        }
    }
    std::string take_string() {
        const uint64_t n = take<uint64_t>();
        need(n);
        std::string s(reinterpret_cast<const char *>(base_ + pos_), size_t(n));
        pos_ += n;
        return s;
    }
    // value of type t: integers kept (as u64), strings kept, the rest skipped
    void take_value(uint32_t t, const std::string &key, bool keep) {
        static const uint64_t widths[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
        if (t == 8) {
            std::string s = take_string();
            if (keep) {
                strings_[key] = std::move(s);
            }
        } else if (t == 9) {
            const uint32_t et = take<uint32_t>();
            const uint64_t n = take<uint64_t>();
            for (uint64_t i = 0; i < n; ++i) {
                take_value(et, key, false);
            }
        } else if (t < 13) {
            const uint64_t w = widths[t];
            need(w);
            uint64_t v = 0;
            std::memcpy(&v, base_ + pos_, size_t(w));
            pos_ += w;
            if (keep && t != 6 && t != 12) {
                ints_[key] = v;
            }
        } else {
            throw std::string("GGUF metadata value of unknown type");
        }
    }
    void parse() {
        if (std::memcmp(base_, "GGUF", 4) != 0) {
            throw std::string("not a GGUF file");
        }
        pos_ = 4;
        const uint32_t version = take<uint32_t>();
        if (version != 3) {
            throw std::string("GGUF version ") + std::to_string(version) + " (3 expected)";
        }
        const uint64_t n_tensors = take<uint64_t>();
        const uint64_t n_kv = take<uint64_t>();
        for (uint64_t i = 0; i < n_kv; ++i) {
            const std::string key = take_string();
            take_value(take<uint32_t>(), key, true);
        }
        struct Info {
            std::string name;
            GgufTensorView v;
            uint64_t offset;
        };
        std::vector<Info> infos(n_tensors);
        for (Info &in : infos) {
            in.name = take_string();
            const uint32_t dims = take<uint32_t>();
            if (dims > 4) {
                throw std::string("GGUF tensor rank above 4: ") + in.name;
            }
            uint64_t elems = 1;
            for (uint32_t d = 0; d < dims; ++d) {
                in.v.shape.push_back(take<uint64_t>());
                elems *= in.v.shape.back();
            }
            in.v.type = take<uint32_t>();
            in.offset = take<uint64_t>();
            if (in.v.type == kGgufF32) {
                in.v.bytes = 4 * elems;
            } else if (in.v.type == kGgufMxfp4) {
                in.v.bytes = elems / 32 * 17;
            } else {
                in.v.bytes = 0;  // not read by the MoE path
            }
        }
        const uint64_t align = ints_.count("general.alignment") ? ints_["general.alignment"] : 32;
        const uint64_t data = (pos_ + align - 1) / align * align;
        for (Info &in : infos) {
            if (data + in.offset > size_ || in.v.bytes > size_ - data - in.offset) {
                throw std::string("GGUF tensor outside the file: ") + in.name;
            }
            in.v.data = base_ + data + in.offset;
            tensors_[in.name] = in.v;
        }
    }

    int fd_ = -1;
    size_t size_ = 0;
    const uint8_t *base_ = nullptr;
    uint64_t pos_ = 0;
    std::map<std::string, uint64_t> ints_;
    std::map<std::string, std::string> strings_;
    std::map<std::string, GgufTensorView> tensors_;
};

void require_shape(const GgufTensorView &t, uint32_t type, std::vector<uint64_t> shape, const std::string &name) {
    if (t.type != type || t.shape != shape) {
        throw std::string("unexpected type or shape for GGUF tensor ") + name;
    }
}

} // namespace

extern "C" {

int ttl_requant_gpu(const char *gguf_path, const char *ttq_path, int layer_begin, int layer_end, int device) {
    if (!gguf_path || !ttq_path) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, "null path");
    }
    ttl_ttq_writer *w = nullptr;
    uint8_t *d_in = nullptr, *d_out = nullptr;
    std::vector<uint8_t> packed;
    int rc = TTL_OK;
    try {
        GgufMap g(gguf_path);
        if (g.string("general.architecture") != "gpt-oss") {
            throw std::string("model architecture is not gpt-oss");
        }
        const uint64_t layers = g.integer("gpt-oss.block_count");
        const uint64_t experts = g.integer("gpt-oss.expert_count");
        if (!((layers == 24 && experts == 32) || (layers == 36 && experts == 128)) ||
            g.integer("gpt-oss.embedding_length") != kDim) {
            throw std::string("only gpt-oss-20b and gpt-oss-120b are supported");
        }
        if (layer_end < 0) {
            layer_end = int(layers);
        }
        if (layer_begin < 0 || layer_begin > layer_end || uint64_t(layer_end) > layers) {
            throw std::string("bad layer range");
        }
        const uint64_t E = experts;
        const int n_layers = layer_end - layer_begin;
        // every tensor is checked before the output file or the GPU is touched
        for (int l = layer_begin; l < layer_end; ++l) {
            const std::string p = "blk." + std::to_string(l) + ".";
            require_shape(g.tensor(p + "ffn_gate_inp.weight"), kGgufF32, {kDim, E}, p + "ffn_gate_inp.weight");
            require_shape(g.tensor(p + "ffn_gate_inp.bias"), kGgufF32, {E}, p + "ffn_gate_inp.bias");
            for (const char *m : {"gate", "up", "down"}) {
                const std::string n = p + "ffn_" + m + "_exps.";
                require_shape(g.tensor(n + "weight"), kGgufMxfp4, {kDim, kDim, E}, n + "weight");
                require_shape(g.tensor(n + "bias"), kGgufF32, {kDim, E}, n + "bias");
            }
        }
        // per layer: router weight + bias, three expert matrices + their biases
        rc = ttl_ttq_open(ttq_path, layers == 24 ? 20 : 120, uint32_t(layers), uint32_t(E), uint32_t(8 * n_layers),
                          &w);
        if (rc) {
            return rc;
        }
        if (device >= 0 && cudaSetDevice(device) != cudaSuccess) {
            throw std::string("cannot select device");
        }
        const size_t gguf_bytes = size_t(E) * kDim * (kDim / 32) * 17;
        const size_t packed_bytes = ttl_packed_bytes(E);
        if (cudaMalloc(&d_in, gguf_bytes) != cudaSuccess || cudaMalloc(&d_out, packed_bytes) != cudaSuccess) {
            throw std::string("device allocation failed");
        }
        packed.resize(packed_bytes);
        for (int l = layer_begin; l < layer_end; ++l) {
            const std::string p = "blk." + std::to_string(l) + ".";
            auto f32 = [&](const std::string &suffix, std::vector<uint64_t> shape) {
                const std::string name = p + suffix;
                const GgufTensorView &t = g.tensor(name);
                require_shape(t, kGgufF32, shape, name);
                rc = ttl_ttq_add(w, name.c_str(), TTL_TTQ_FORMAT_F32, uint32_t(shape.size()), shape.data(), t.data,
                                 t.bytes);
                if (rc) {
                    throw std::string(ttl_moe_last_error(nullptr));
                }
            };
            f32("ffn_gate_inp.weight", {kDim, E});
            f32("ffn_gate_inp.bias", {E});
            for (const char *m : {"gate", "up", "down"}) {
                const std::string name = p + "ffn_" + m + "_exps.weight";
                const GgufTensorView &t = g.tensor(name);
                require_shape(t, kGgufMxfp4, {kDim, kDim, E}, name);
                if (cudaMemcpy(d_in, t.data, gguf_bytes, cudaMemcpyHostToDevice) != cudaSuccess) {
                    throw std::string("weight copy failed");
                }
                rc = ttl_pack_mxfp4(d_in, E, d_out, -1);
                if (rc) {
                    throw std::string(ttl_moe_last_error(nullptr));
                }
                if (cudaMemcpy(packed.data(), d_out, packed_bytes, cudaMemcpyDeviceToHost) != cudaSuccess) {
                    throw std::string("packed copy failed");
                }
                const uint64_t shape[3] = {kDim, kDim, E};
                const std::string rec = name + ".mxfp4gpu";
                rc = ttl_ttq_add(w, rec.c_str(), TTL_TTQ_FORMAT_MXFP4_GPU, 3, shape, packed.data(), packed_bytes);
                if (rc) {
                    throw std::string(ttl_moe_last_error(nullptr));
                }
                f32(std::string("ffn_") + m + "_exps.bias", {kDim, E});
            }
        }
        rc = ttl_ttq_finish(w);
        if (rc) {
            throw std::string(ttl_moe_last_error(nullptr));
        }
    } catch (const std::string &e) {
        rc = ttl::fail(nullptr, rc ? rc : TTL_ERR_IO, "requant: " + e);
    }
    if (w) {
        ttl_ttq_close(w);  // removes an unfinished file
    }
    cudaFree(d_in);
    cudaFree(d_out);
    return rc;
}

} // extern "C"
