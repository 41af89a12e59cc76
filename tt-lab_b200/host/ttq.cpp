// ttq.cpp -- TTQ container writer for the GPU weight layout (requant --cuda).
//
// The container is tt-lab's own TTLBQNT1 format, kept byte-compatible so the
// existing reader (TtqFile, src/tt_backend.cpp:315-445) parses it: a 56-byte
// header (src/requant.h:31-44), a directory of 184-byte records
// (src/requant.h:46-53), then 64-byte aligned payloads (src/requant.h:17-18).
// The write is atomic like TtqOutput (src/requant.cpp:23-68): everything goes
// to a mkstemp file beside the target, the header and directory are rewritten
// at the end, and rename() replaces the target; any failure removes the
// temporary file.  MXFP4 expert tensors use the new format id 6
// (TTL_TTQ_FORMAT_MXFP4_GPU), produced by ttl_pack_mxfp4.
#include <cerrno>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include <unistd.h>

#include "../csrc/internal.h"
#include "ttl_moe.h"

namespace {

struct TtqHeader {
    char magic[8];
    uint32_t version;
    uint32_t model;
    uint32_t tensor_count;
    uint32_t reserved;
    uint64_t directory_offset;
    uint64_t data_offset;
    uint32_t layer_count;
    uint32_t expert_count;
    uint32_t dim;
    uint32_t vocab;
};
static_assert(sizeof(TtqHeader) == 56, "TTQ header layout");

struct TtqRecord {
    char name[128];
    uint32_t format;
    uint32_t rank;
    uint64_t shape[4];
    uint64_t offset;
    uint64_t size;
};
static_assert(sizeof(TtqRecord) == 184, "TTQ record layout");

constexpr uint64_t kAlign = 64;

} // namespace

struct ttl_ttq_writer {
    std::string path;
    std::string temporary;
    std::FILE *stream = nullptr;
    TtqHeader header{};
    std::vector<TtqRecord> records;
    size_t added = 0;
    bool finished = false;
};

namespace {

int io_fail(const std::string &what) {
    return ttl::fail(nullptr, TTL_ERR_IO, what + ": " + std::strerror(errno));
}

bool write_at(std::FILE *f, uint64_t offset, const void *data, size_t size) {
    return std::fseek(f, long(offset), SEEK_SET) == 0 && std::fwrite(data, 1, size, f) == size;
}

} // namespace

extern "C" {

int ttl_ttq_open(const char *path, uint32_t model, uint32_t layers, uint32_t experts, uint32_t tensor_count,
                 ttl_ttq_writer **writer_out) {
    if (!path || !writer_out) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, "null path or writer");
    }
    *writer_out = nullptr;
    if (!((model == 20 && layers == 24 && experts == 32) || (model == 120 && layers == 36 && experts == 128))) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, "only gpt-oss-20b and gpt-oss-120b are supported by requant");
    }
    ttl_ttq_writer *w = new ttl_ttq_writer();
    w->path = path;
    w->temporary = w->path + ".tmp.XXXXXX";
    const int fd = mkstemp(w->temporary.data());
    if (fd < 0) {
        const int rc = io_fail("cannot create temporary TTQ file beside " + w->path);
        w->temporary.clear();
        delete w;
        return rc;
    }
    w->stream = fdopen(fd, "wb");
    if (!w->stream) {
        const int rc = io_fail("cannot open temporary TTQ stream");
        close(fd);
        unlink(w->temporary.c_str());
        w->temporary.clear();
        delete w;
        return rc;
    }
    const char magic[8] = {'T', 'T', 'L', 'B', 'Q', 'N', 'T', '1'};
    std::memcpy(w->header.magic, magic, sizeof(magic));
    w->header.version = 1;
    w->header.model = model;
    w->header.tensor_count = tensor_count;
    w->header.directory_offset = sizeof(TtqHeader);
    w->header.data_offset =
        (sizeof(TtqHeader) + uint64_t(tensor_count) * sizeof(TtqRecord) + kAlign - 1) & ~(kAlign - 1);
    w->header.layer_count = layers;
    w->header.expert_count = experts;
    w->header.dim = 2880;
    w->header.vocab = 201088;
    w->records.assign(tensor_count, TtqRecord{});
    std::vector<char> zeros(w->header.data_offset, 0);
    if (!write_at(w->stream, 0, zeros.data(), zeros.size())) {
        const int rc = io_fail("cannot write TTQ header");
        ttl_ttq_close(w);
        return rc;
    }
    *writer_out = w;
    return TTL_OK;
}

int ttl_ttq_add(ttl_ttq_writer *w, const char *name, uint32_t format, uint32_t rank, const uint64_t *shape,
                const void *payload, uint64_t size) {
    if (!w || !name || (!payload && size) || (rank && !shape)) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, "null argument");
    }
    if (w->finished || w->added >= w->records.size()) {
        return ttl::fail(nullptr, TTL_ERR_STATE, "more TTQ records than announced");
    }
    if (std::strlen(name) >= sizeof(TtqRecord::name)) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, std::string("TTQ tensor name is too long: ") + name);
    }
    if (rank > 4) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, std::string("TTQ tensor rank is too large: ") + name);
    }
    if (std::fseek(w->stream, 0, SEEK_END) != 0) {
        return io_fail("cannot seek TTQ file");
    }
    const long end = std::ftell(w->stream);
    if (end < 0) {
        return io_fail("cannot tell TTQ file");
    }
    const uint64_t offset = (uint64_t(end) + kAlign - 1) & ~(kAlign - 1);
    static const char pad[kAlign] = {};
    if (offset > uint64_t(end) && std::fwrite(pad, 1, offset - uint64_t(end), w->stream) != offset - uint64_t(end)) {
        return io_fail("cannot align TTQ payload");
    }
    if (size && std::fwrite(payload, 1, size, w->stream) != size) {
        return io_fail(std::string("cannot write TTQ payload ") + name);
    }
    TtqRecord &r = w->records[w->added++];
    std::memcpy(r.name, name, std::strlen(name));
    r.format = format;
    r.rank = rank;
    for (uint32_t i = 0; i < rank; ++i) {
        r.shape[i] = shape[i];
    }
    r.offset = offset;
    r.size = size;
    return TTL_OK;
}

int ttl_ttq_finish(ttl_ttq_writer *w) {
    if (!w || w->finished) {
        return ttl::fail(nullptr, TTL_ERR_ARGUMENT, "bad writer");
    }
    if (w->added != w->records.size()) {
        return ttl::fail(nullptr, TTL_ERR_STATE, "internal TTQ record count mismatch");
    }
    if (!write_at(w->stream, 0, &w->header, sizeof(w->header)) ||
        (!w->records.empty() &&
         !write_at(w->stream, w->header.directory_offset, w->records.data(), w->records.size() * sizeof(TtqRecord)))) {
        return io_fail("cannot write TTQ directory");
    }
    const int closed = std::fclose(w->stream);
    w->stream = nullptr;
    if (closed != 0) {
        return io_fail("cannot close TTQ file " + w->path);
    }
    if (std::rename(w->temporary.c_str(), w->path.c_str()) != 0) {
        return io_fail("cannot replace TTQ file " + w->path);
    }
    w->temporary.clear();
    w->finished = true;
    return TTL_OK;
}

void ttl_ttq_close(ttl_ttq_writer *w) {
    if (!w) {
        return;
    }
    if (w->stream) {
        std::fclose(w->stream);
    }
    if (!w->temporary.empty()) {
        unlink(w->temporary.c_str());
    }
    delete w;
}

} // extern "C"
