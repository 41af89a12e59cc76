// ttq_shim.cpp -- tt-lab's own TTQ reader (TtqFile, src/tt_backend.cpp:315-445)
// on files the backend writes.  TEST INFRASTRUCTURE ONLY.
//
// TtqFile is internal to tt_backend.cpp, so this translation unit includes
// that file as it is (compiled unmodified, with the reference's flags); the
// BRISC firmware it embeds is SFPI-generated code that cannot be built here,
// and oracle/Makefile supplies a one-byte placeholder for it (the reader
// never touches the firmware).  Exposed as a C API for the tests.
#include "tt_backend.cpp"

namespace {
thread_local std::string g_ttq_error;
}

extern "C" {

const char *tref_ttq_last_error() {
    return g_ttq_error.c_str();
}

// Opens `path` with TtqFile; the handle is freed by tref_ttq_close.
void *tref_ttq_open(const char *path) {
    try {
        return new TtqFile(path);
    } catch (const std::exception &e) {
        g_ttq_error = e.what();
        return nullptr;
    }
}

void tref_ttq_close(void *f) {
    delete static_cast<TtqFile *>(f);
}

size_t tref_ttq_count(void *f) {
    return static_cast<TtqFile *>(f)->tensors().size();
}

size_t tref_ttq_layers(void *f) {
    return static_cast<TtqFile *>(f)->layer_count();
}

// Record i: name (<= 127 chars + NUL into name[128]), format, rank, shape[4],
// payload pointer and size as TtqFile exposes them.
int tref_ttq_record(void *f, size_t i, char *name, uint32_t *format, uint32_t *rank, uint64_t *shape,
                    const void **data, uint64_t *size) {
    auto &ts = static_cast<TtqFile *>(f)->tensors();
    if (i >= ts.size()) {
        return -1;
    }
    const TtqTensor &t = ts[i];
    std::snprintf(name, 128, "%s", t.name.c_str());
    *format = t.format;
    *rank = uint32_t(t.shape.size());
    for (size_t d = 0; d < 4; ++d) {
        shape[d] = d < t.shape.size() ? t.shape[d] : 0;
    }
    *data = t.data;
    *size = t.size;
    return 0;
}

// TtqFile::tensor(name): the payload of a named record, or NULL.
const void *tref_ttq_find(void *f, const char *name, uint64_t *size) {
    try {
        const TtqTensor &t = static_cast<TtqFile *>(f)->tensor(name);
        *size = t.size;
        return t.data;
    } catch (const std::exception &e) {
        g_ttq_error = e.what();
        return nullptr;
    }
}

} // extern "C"
