// moe.cu -- the ttl_moe handle: start-up, weight upload, and the decode,
// prefill and layer-stack entry points of include/ttl_moe.h.
//
// One handle drives one GPU.  Expert parallelism (world > 1) runs one process
// per GPU; each rank holds experts [rank*E/world, (rank+1)*E/world).  The
// router is replicated (it is 0.7% of a layer's bytes) so every rank derives
// the same top-4 for the same token.  Decode: the ranks add their partial
// outputs inside the persistent kernel, through exchange buffers they map from
// each other's CUDA IPC handles (NVLink peer stores); per-layer kernels with
// an NCCL all-reduce stand in when that mapping is unavailable.  Prefill: each
// rank passes its own tokens, which go to their experts' owners and come back
// as weighted rows (NCCL send/recv, prefill_ep.cu).
#include <cuda.h>  // CUtensorMap types; the encoder is resolved through the runtime
#include <cuda_runtime.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "nccl_dl.h"

namespace ttl {
void configure_decode_kernels();
void configure_prefill_kernels();
void configure_prefill_tc();
} // namespace ttl

using namespace ttl;

namespace {

struct LayerStore {
    bool uploaded = false;
    float *router_w = nullptr;
    float *router_b = nullptr;
    float *norm_w = nullptr;
    uint8_t *gate = nullptr;
    uint8_t *up = nullptr;
    uint8_t *down = nullptr;
    float *gate_b = nullptr;
    float *up_b = nullptr;
    float *down_b = nullptr;
};

constexpr size_t kMaxForwardGraphs = 64;       // captured forward graphs kept per handle
constexpr size_t kForwardStagingTokens = 256;  // ttl_moe_forward's device rows (at least)

struct GraphKey {
    const void *x;
    const void *y;
    size_t tokens;
    int begin;
    int end;
    bool operator<(const GraphKey &o) const {
        return std::tie(x, y, tokens, begin, end) < std::tie(o.x, o.y, o.tokens, o.begin, o.end);
    }
};

} // namespace

struct ttl_moe {
    ttl_moe_config cfg{};
    int device = 0;
    int sms = 148;
    cudaStream_t stream = nullptr;
    std::string error;
    int expert_begin = 0;
    int expert_count = 0;
    std::vector<LayerStore> layers;
    std::vector<void *> allocations;
    uint8_t *staging = nullptr;  // one GGUF expert tensor (this rank's experts)
    size_t staging_bytes = 0;
    DecodeWork dw{};
    PrefillWork pw{};
    float *d_x = nullptr;        // [max(1, max_tokens)][2880]
    float *d_y = nullptr;
    float *d_fwd = nullptr;      // forward staging for host calls [fwd_cap][2880], allocated at create
    size_t fwd_cap = 0;
    float *d_ones = nullptr;
    uint32_t *d_status = nullptr;
    unsigned long long *d_counters = nullptr;
    uint64_t launches = 0;
    ncclComm_t comm = nullptr;   // nonblocking: every wait on it is bounded by timeout_ms
    // Expert-parallel fault state.  The ranks' kernels meet on tags derived
    // from per-rank bases (d_seq, ep.seq), so after any failed call on a
    // multi-rank handle the ranks may disagree about them: ep_fault is set,
    // and compute calls are refused until every rank has run ttl_moe_resync.
    // comm_dead: the communicator was aborted (a collective missed its deadline).
    bool ep_fault = false;
    bool comm_dead = false;
    uint32_t timeout_ms = 60000;     // host-side bound on waits for the stream and for NCCL
    cudaEvent_t wait_ev = nullptr;   // recorded for the bounded stream wait (world > 1)
    uint32_t *d_sync = nullptr;      // [4] resync scratch (world > 1)
    struct ForwardGraph {
        cudaGraphExec_t exec;
        uint64_t kernels;   // kernels per replay
        uint64_t last_use;  // graph_clock of the last replay
    };
    std::map<GraphKey, ForwardGraph> graphs;  // at most kMaxForwardGraphs, least recently used evicted
    uint64_t graph_clock = 0;
    // the blocking single-layer decode (ttl_moe_decode): pinned staging of its
    // input and outputs, and one captured graph per layer (copies in, the
    // persistent kernel, copies out with the status word)
    // (the device copy of DecodeBlock holds the handle's status word, so one
    // copy brings back the output, the top-4 and the status)
    struct DecodeBlock {
        float y[kDim];
        int32_t idx[4];
        float w[4];
        uint32_t status;
        uint32_t pad[3];
    };
    struct DecodePin {
        float x[kDim];
        DecodeBlock out;
    };
    DecodePin *pin = nullptr;        // pinned host staging, allocated at create
    // the decode server (ttl_moe_serve): a resident launch fed through a
    // mailbox in mapped pinned memory
    DecodeMailbox *mbox = nullptr;      // host address
    DecodeMailbox *mbox_dev = nullptr;  // the same memory as the device addresses it
    float *d_srv_x = nullptr;           // [2880] the request's input on the device
    unsigned long long *d_go = nullptr; // the server's per-step go word
    uint32_t serve_idle_us = 0;         // 0: no server
    bool serving = false;               // a server launch may still be on the stream
    uint32_t req = 0;                   // requests submitted to the mailbox
    uint32_t mbox_base = 0;             // requests answered before the current server launch
    DecodeBlock *d_dblk = nullptr;   // device side
    std::map<int, std::pair<cudaGraphExec_t, uint64_t>> decode_graphs;  // per layer, captured at upload
    bool profile = false;
    int profile_layers = 0;        // layers covered by the recorded events
    std::vector<cudaEvent_t> events;  // [layers][4]
    // persistent decode kernel
    unsigned long long *d_part_gu = nullptr;  // tagged tile partials, [2] x gate/up and down
    unsigned long long *d_part_dn = nullptr;
    unsigned long long *d_rpt = nullptr;  // tagged router sums per down tile
    unsigned long long *d_rlog = nullptr;  // tagged (logit, bound) pairs of the exact-router steps
    unsigned *d_cnt = nullptr;        // [5] gate/up tiles reduced per expert slot, down tiles with y and B written
    uint8_t *d_bdown = nullptr;
    uint8_t *d_sfb_down = nullptr;
    uint8_t *d_bnext = nullptr;       // next step's gate/up B operand (written by the down epilogues)
    uint8_t *d_bnext_code = nullptr;
    uint32_t *d_seq = nullptr;        // [2] tag base of the next launch and its finish count
    // expert parallelism inside the persistent kernel (world > 1)
    unsigned long long *d_xch = nullptr;         // this rank's exchange buffer [2][world][kXchRow]
    unsigned long long **d_xch_peers = nullptr;  // [world] every rank's buffer as this GPU addresses it
    void *xch_open[kMaxWorld] = {};              // the peers' buffers, opened from their IPC handles
    bool xch_ready = false;                      // every rank mapped every buffer
    // expert-parallel prefill (world > 1): the own tokens' routing, the
    // dispatch plan, and the receive blocks every rank maps (prefill_ep.cu)
    struct {
        int32_t *own_idx = nullptr;    // [T][4] top-4 of this rank's own tokens
        float *own_w = nullptr;        // [T][4]
        float *own_logits = nullptr;   // [T][E]
        int32_t *tok_off = nullptr;    // [T][world] row of each own token in each destination's region (-1: none)
        int32_t *cnt = nullptr;        // [world] rows sent to each rank
        int32_t *rcnt = nullptr;       // [world] rows received from each rank (this call)
        unsigned *arrive = nullptr;    // [2] grid arrival counters of the send and back kernels
        void *inbox = nullptr;         // this rank's receive block (IPC allocation), ep_inbox_bytes
        int cap = 0;                   // rows per source region = max_tokens
        EpPeers peers{};               // every rank's block as this GPU addresses it
        void *open[kMaxWorld] = {};    // the peers' blocks, opened from their IPC handles
        bool mapped = false;           // every rank mapped every block
        uint32_t seq = 0;              // tag of the last call (agreed by every rank)
    } ep;
    StackLayer *d_layers = nullptr;   // [layers]
    TmaDesc *d_tma = nullptr;         // [layers][kTmaCount] tensor maps of the packed matrices
    uint32_t *d_pack_flags = nullptr; // packer flags of the last upload
    std::vector<StackLayer> host_layers;
    double *d_acc = nullptr;          // [2][kMaxExperts + 1]
    unsigned *d_barrier = nullptr;    // [2]
    cudaEvent_t stack_ev[2] = {nullptr, nullptr};
    bool stack_profiled = false;
    int stack_steps = 0;              // (token, layer) steps of the profiled launch
    unsigned long long *d_trace = nullptr;  // phase stamps (ttl_moe_trace)
    int trace_steps = 0;
    float *log_y = nullptr;           // step log (ttl_moe_record): caller's device buffers
    int32_t *log_idx = nullptr;
    float *log_w = nullptr;
    int log_steps = 0;
};

namespace ttl {

std::string &thread_error() {
    thread_local std::string message;
    return message;
}

int fail(ttl_moe *handle, int code, const std::string &message) {
    if (handle) {
        handle->error = message;
        if (handle->cfg.world > 1) {
            handle->ep_fault = true;
        }
    } else {
        thread_error() = message;
    }
    return code;
}

const char *handle_error(const ttl_moe *handle) {
    return handle ? handle->error.c_str() : thread_error().c_str();
}

bool is_device_pointer(const void *p) {
    if (!p) {
        return false;
    }
    cudaPointerAttributes attr{};
    if (cudaPointerGetAttributes(&attr, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    return attr.type == cudaMemoryTypeDevice || attr.type == cudaMemoryTypeManaged;
}

} // namespace ttl

namespace {

int alloc(ttl_moe *h, void **p, size_t bytes) {
    if (bytes == 0) {
        *p = nullptr;
        return TTL_OK;
    }
    const cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) {
        return fail(h, TTL_ERR_CUDA, "cudaMalloc(" + std::to_string(bytes) + "): " + cudaGetErrorString(e));
    }
    h->allocations.push_back(*p);
    return TTL_OK;
}

template <class T> int alloc_n(ttl_moe *h, T **p, size_t n) {
    return alloc(h, reinterpret_cast<void **>(p), n * sizeof(T));
}

LayerDev layer_view(const ttl_moe *h, int layer) {
    const LayerStore &s = h->layers[size_t(layer)];
    LayerDev L;
    L.router_w = s.router_w;
    L.router_b = s.router_b;
    L.norm_w = s.norm_w ? s.norm_w : h->d_ones;
    L.gate = s.gate;
    L.up = s.up;
    L.down = s.down;
    L.gate_b = s.gate_b;
    L.up_b = s.up_b;
    L.down_b = s.down_b;
    return L;
}

DecodeShape decode_shape(const ttl_moe *h) {
    return DecodeShape{int(h->cfg.experts), h->expert_begin, h->expert_count, h->sms};
}

int check_layer(ttl_moe *h, int layer) {
    if (layer < 0 || layer >= int(h->cfg.layers)) {
        return fail(h, TTL_ERR_ARGUMENT, "layer " + std::to_string(layer) + " out of range");
    }
    if (!h->layers[size_t(layer)].uploaded) {
        return fail(h, TTL_ERR_STATE, "layer " + std::to_string(layer) + " was not uploaded");
    }
    return TTL_OK;
}

int set_device(ttl_moe *h) {
    TTL_TRY_CUDA(h, cudaSetDevice(h->device));
    return TTL_OK;
}

using Clock = std::chrono::steady_clock;

// Aborts the communicator; the handle then refuses every compute call and
// must be destroyed.
int abort_comm(ttl_moe *h, const std::string &why) {
    if (h->comm) {
        nccl(nullptr)->CommAbort(h->comm);
        h->comm = nullptr;
    }
    h->comm_dead = true;
    return fail(h, TTL_ERR_NCCL, why + "; the communicator was aborted (destroy the handle)");
}

// The communicator is nonblocking: a call that answers ncclInProgress has
// completed once ncclCommGetAsyncError stops answering it.  Bounded by the
// handle's deadline; an asynchronous error or the deadline aborts it.
int comm_settle(ttl_moe *h, const char *what) {
    const NcclApi *api = nccl(nullptr);
    const auto deadline = Clock::now() + std::chrono::milliseconds(h->timeout_ms);
    for (;;) {
        ncclResult_t state = ncclSuccess;
        const ncclResult_t r = api->CommGetAsyncError(h->comm, &state);
        if (r != ncclSuccess) {
            state = r;
        }
        if (state == ncclSuccess) {
            return TTL_OK;
        }
        if (state != ncclInProgress) {
            return abort_comm(h, std::string(what) + ": " + api->GetErrorString(state));
        }
        if (Clock::now() > deadline) {
            return abort_comm(h, std::string(what) + ": not complete after " + std::to_string(h->timeout_ms) + " ms");
        }
        std::this_thread::yield();
    }
}

int nccl_check(ttl_moe *h, ncclResult_t r, const char *what) {
    if (r == ncclInProgress) {
        return comm_settle(h, what);
    }
    if (r != ncclSuccess) {
        const NcclApi *api = nccl(nullptr);
        return fail(h, TTL_ERR_NCCL, std::string(what) + ": " + (api ? api->GetErrorString(r) : "nccl unavailable"));
    }
    return TTL_OK;
}

// Waits for everything enqueued on the handle's stream.  A multi-rank handle
// waits by polling an event, bounded by its deadline, and watches its
// communicator meanwhile: an NCCL error or the deadline aborts it, after
// which the stream gets one more deadline to drain.  The kernels' own waits
// on peers are bounded on the device (2 s) and end in a status word.
int stream_wait(ttl_moe *h) {
    if (h->cfg.world == 1 || !h->wait_ev) {
        TTL_TRY_CUDA(h, cudaStreamSynchronize(h->stream));
        return TTL_OK;
    }
    TTL_TRY_CUDA(h, cudaEventRecord(h->wait_ev, h->stream));
    const NcclApi *api = nccl(nullptr);
    auto deadline = Clock::now() + std::chrono::milliseconds(h->timeout_ms);
    int rc = TTL_OK;
    for (;;) {
        const cudaError_t q = cudaEventQuery(h->wait_ev);
        if (q == cudaSuccess) {
            return rc;
        }
        if (q != cudaErrorNotReady) {
            return fail(h, TTL_ERR_CUDA, std::string("stream wait: ") + cudaGetErrorString(q));
        }
        if (h->comm) {
            ncclResult_t state = ncclSuccess;
            if (api->CommGetAsyncError(h->comm, &state) == ncclSuccess && state != ncclSuccess &&
                state != ncclInProgress) {
                rc = abort_comm(h, std::string("NCCL: ") + api->GetErrorString(state));
                deadline = Clock::now() + std::chrono::milliseconds(h->timeout_ms);
            }
        }
        if (Clock::now() > deadline) {
            if (!h->comm) {
                return rc ? rc : fail(h, TTL_ERR_NCCL, "the stream did not drain within the deadline");
            }
            rc = abort_comm(h, "stream not finished after " + std::to_string(h->timeout_ms) + " ms");
            deadline = Clock::now() + std::chrono::milliseconds(h->timeout_ms);
        }
        std::this_thread::yield();
    }
}

// Compute calls on a multi-rank handle are refused after a failure until the
// ranks have agreed again (ttl_moe_resync), or for good once the
// communicator was aborted.
int ep_ready(ttl_moe *h) {
    if (h->cfg.world == 1) {
        return TTL_OK;
    }
    if (h->comm_dead) {
        return fail(h, TTL_ERR_NCCL, "the communicator was aborted after a failure; destroy the handle");
    }
    if (h->ep_fault) {
        return fail(h, TTL_ERR_STATE,
                    "an earlier call failed on this expert-parallel handle; every rank must call ttl_moe_resync "
                    "before the next compute call");
    }
    return TTL_OK;
}

// Sum of the ranks' partial outputs, in place on the handle's stream.
int allreduce(ttl_moe *h, float *buf, size_t n) {
    if (h->cfg.world <= 1) {
        return TTL_OK;
    }
    return nccl_check(h, nccl(nullptr)->AllReduce(buf, buf, n, ncclFloat32, ncclSum, h->comm, h->stream),
                      "ncclAllReduce");
}

// The persistent decode kernel serves world == 1, and world > 1 once every
// rank's exchange buffer is mapped on every rank (tensor-core kernel only);
// otherwise decode runs per layer with an NCCL all-reduce.
bool stack_path(const ttl_moe *h) {
    return h->cfg.world == 1 || h->xch_ready;
}

// Peer memory for expert parallelism: this rank's exchange buffer (the
// persistent decode kernel's partial rows) and, with a prefill capacity, its
// receive block (prefill_ep.cu); the IPC handles of all ranks gathered over
// NCCL, the peers' allocations opened (peer access over NVLink), and tables
// of them on the device.  The ranks then agree (NCCL min) that every one of
// them succeeded, so all take the same paths.  Returns TTL_OK either way; if
// any rank could not map, decode runs per layer with an NCCL all-reduce on
// every rank and prefill is refused.
int setup_exchange(ttl_moe *h) {
    const int W = int(h->cfg.world);
    const int R = int(h->cfg.rank);
    const NcclApi *api = nccl(nullptr);
    int ok = 1;
    uint8_t *d_handles = nullptr;
    int *d_ok = nullptr;
    constexpr size_t kHandle = sizeof(cudaIpcMemHandle_t);
    int rc = alloc_n(h, &h->d_xch, xch_words(W));
    rc = rc ? rc : alloc_n(h, &h->d_xch_peers, size_t(W));
    rc = rc ? rc : alloc_n(h, &d_handles, size_t(W) * 2 * kHandle);
    rc = rc ? rc : alloc_n(h, &d_ok, 1);
    if (rc) {
        return rc;
    }
    cudaIpcMemHandle_t mine[2] = {};
    if (cudaMemset(h->d_xch, 0, xch_words(W) * sizeof(unsigned long long)) != cudaSuccess ||
        cudaIpcGetMemHandle(&mine[0], h->d_xch) != cudaSuccess ||
        (h->ep.inbox && cudaIpcGetMemHandle(&mine[1], h->ep.inbox) != cudaSuccess)) {
        ok = 0;
        cudaGetLastError();
    }
    TTL_TRY_CUDA(h, cudaMemcpy(d_handles + size_t(R) * 2 * kHandle, mine, 2 * kHandle, cudaMemcpyHostToDevice));
    rc = nccl_check(h, api->AllGather(d_handles + size_t(R) * 2 * kHandle, d_handles, 2 * kHandle, ncclUint8,
                                      h->comm, h->stream),
                    "ncclAllGather");
    rc = rc ? rc : stream_wait(h);
    if (rc) {
        return rc;
    }
    std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(2 * W));
    TTL_TRY_CUDA(h, cudaMemcpy(all.data(), d_handles, size_t(W) * 2 * kHandle, cudaMemcpyDeviceToHost));
    std::vector<unsigned long long *> ptrs(static_cast<size_t>(W), nullptr);
    for (int r = 0; r < W && ok; ++r) {
        if (r == R) {
            ptrs[size_t(r)] = h->d_xch;
            h->ep.peers.base[r] = h->ep.inbox;
            continue;
        }
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, all[size_t(2 * r)], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            ok = 0;
            cudaGetLastError();
            break;
        }
        h->xch_open[r] = p;
        ptrs[size_t(r)] = static_cast<unsigned long long *>(p);
        if (h->ep.inbox) {
            void *q = nullptr;
            if (cudaIpcOpenMemHandle(&q, all[size_t(2 * r + 1)], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
                ok = 0;
                cudaGetLastError();
                break;
            }
            h->ep.open[r] = q;
            h->ep.peers.base[r] = q;
        }
    }
    TTL_TRY_CUDA(h, cudaMemcpy(h->d_xch_peers, ptrs.data(), size_t(W) * sizeof(void *), cudaMemcpyHostToDevice));
    TTL_TRY_CUDA(h, cudaMemcpy(d_ok, &ok, sizeof(int), cudaMemcpyHostToDevice));
    rc = nccl_check(h, api->AllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, h->comm, h->stream), "ncclAllReduce");
    rc = rc ? rc : stream_wait(h);
    if (rc) {
        return rc;
    }
    TTL_TRY_CUDA(h, cudaMemcpy(&ok, d_ok, sizeof(int), cudaMemcpyDeviceToHost));
    h->xch_ready = ok != 0;
    h->ep.mapped = ok != 0 && h->ep.inbox != nullptr;
    return TTL_OK;
}

// Enqueues one decode layer: router -> gate/up -> down (+ combine, residual).
int enqueue_decode_layer(ttl_moe *h, int layer, const float *x, int mode, const float *residual, float *out,
                         cudaEvent_t *ev = nullptr) {
    const LayerDev L = layer_view(h, layer);
    const DecodeShape s = decode_shape(h);
    if (ev) {
        cudaEventRecordWithFlags(ev[0], h->stream, cudaEventRecordExternal);
    }
    launch_decode_router(L, h->dw, s, x, mode, h->stream);
    if (ev) {
        cudaEventRecordWithFlags(ev[1], h->stream, cudaEventRecordExternal);
    }
    launch_decode_gateup(L, h->dw, s, h->stream);
    if (ev) {
        cudaEventRecordWithFlags(ev[2], h->stream, cudaEventRecordExternal);
    }
    if (h->cfg.world > 1) {
        launch_decode_down(L, h->dw, s, nullptr, h->dw.partial, h->stream);
        if (ev) {
            cudaEventRecordWithFlags(ev[3], h->stream, cudaEventRecordExternal);
        }
        h->launches += 3;
        int rc = allreduce(h, h->dw.partial, kDim);
        if (rc) {
            return rc;
        }
        if (residual) {
            launch_add(residual, h->dw.partial, out, kDim, h->stream);
        } else {
            TTL_TRY_CUDA(h, cudaMemcpyAsync(out, h->dw.partial, kDim * sizeof(float), cudaMemcpyDeviceToDevice,
                                            h->stream));
        }
        h->launches += 1;
    } else {
        launch_decode_down(L, h->dw, s, residual, out, h->stream);
        if (ev) {
            cudaEventRecordWithFlags(ev[3], h->stream, cudaEventRecordExternal);
        }
        h->launches += 3;
    }
    TTL_TRY_CUDA(h, cudaGetLastError());
    return TTL_OK;
}

static_assert(sizeof(CUtensorMap) == sizeof(TmaDesc) && alignof(TmaDesc) >= 64, "tensor map size");

typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
    static const EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            p = nullptr;
        }
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

// Tensor maps of one layer's packed matrices (order of TmaIndex): the nibble
// rows as bytes, 128-byte x 128-row boxes with 128-byte swizzle (the K-major
// layout of the kind::mxf4 A operand).
int build_layer_maps(ttl_moe *h, const LayerStore &st, TmaDesc *out) {
    const EncodeTiledFn enc = encode_tiled();
    if (!enc) {
        return fail(h, TTL_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    }
    const cuuint64_t experts = cuuint64_t(h->expert_count);
    const cuuint32_t ones[3] = {1, 1, 1};
    CUtensorMap maps[kTmaCount];
    bool ok = true;
    auto weights = [&](int idx, const uint8_t *base) {
        const cuuint64_t dims[3] = {cuuint64_t(kNibbleRowBytes), cuuint64_t(kDim), experts};
        const cuuint64_t strides[2] = {cuuint64_t(kNibbleRowBytes), cuuint64_t(kPackedMatrixBytes)};
        const cuuint32_t box[3] = {128, 128, 1};
        ok = ok && enc(&maps[idx], CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<uint8_t *>(base), dims, strides, box, ones,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    };
    weights(kTmaGate, st.gate);
    weights(kTmaUp, st.up);
    weights(kTmaDown, st.down);
    std::memset(&maps[kTmaRouter], 0, sizeof(maps[kTmaRouter]));
    const int E = int(h->cfg.experts);
    if (E > kRouterMapFirstExpert) {
        const cuuint64_t dims[2] = {cuuint64_t(kDim), cuuint64_t(E)};
        const cuuint64_t strides[1] = {cuuint64_t(kDim) * sizeof(float)};
        const cuuint32_t box[2] = {128, cuuint32_t(E - kRouterMapFirstExpert)};
        ok = ok && enc(&maps[kTmaRouter], CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, st.router_w, dims, strides, box, ones,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
    }
    if (!ok) {
        return fail(h, TTL_ERR_CUDA, "cuTensorMapEncodeTiled rejected a weight tensor map");
    }
    TTL_TRY_CUDA(h, cudaMemcpy(out, maps, sizeof(maps), cudaMemcpyHostToDevice));
    return TTL_OK;
}

int push_layer_descriptor(ttl_moe *h, int layer) {
    const LayerDev L = layer_view(h, layer);
    StackLayer d{L.router_w, L.router_b, L.norm_w, L.gate, L.up, L.down, L.gate_b, L.up_b, L.down_b, nullptr};
    const LayerStore &st = h->layers[size_t(layer)];
    if (st.gate && st.up && st.down) {
        TmaDesc *maps = h->d_tma + size_t(layer) * kTmaCount;
        const int rc = build_layer_maps(h, st, maps);
        if (rc) {
            return rc;
        }
        d.tma = maps;
    }
    h->host_layers[size_t(layer)] = d;
    TTL_TRY_CUDA(h, cudaMemcpy(h->d_layers + layer, &d, sizeof(d), cudaMemcpyHostToDevice));
    return TTL_OK;
}

// One cooperative launch covering `tokens` tokens x layers [begin, end).
int enqueue_stack(ttl_moe *h, int begin, int end, const float *x, float *y, size_t tokens, int mode) {
    StackArgs a{};
    a.layers = h->d_layers;
    a.layer_begin = begin;
    a.layer_end = end;
    a.x = x;
    a.y = y;
    a.tokens = int(tokens);
    a.mode = mode;
    a.row_mask = (mode == 2) ? 0 : 0x7fffffff;
    if (mode == 2) {
        a.mbox = h->mbox_dev;
        a.srv_x = h->d_srv_x;
        a.go = h->d_go;
        a.mbox_base = h->mbox_base;
        a.idle_ns = uint64_t(h->serve_idle_us) * 1000ull;
    }
    a.experts = int(h->cfg.experts);
    a.expert_begin = h->expert_begin;
    a.expert_count = h->expert_count;
    a.acc = h->d_acc;
    a.rlog = h->d_rlog;
    a.hidden = h->dw.hidden;
    a.top_idx = h->dw.top_idx;
    a.top_w = h->dw.top_w;
    a.barrier = h->d_barrier;
    a.status = h->d_status;
    a.counters = h->d_counters;
    a.seq_state = h->d_seq;
    a.rank = int(h->cfg.rank);
    a.world = h->xch_ready ? int(h->cfg.world) : 1;
    a.xch = h->d_xch_peers;
    a.part_gu = h->d_part_gu;
    a.part_dn = h->d_part_dn;
    a.rpt = h->d_rpt;
    a.cnt_b = h->d_cnt;
    a.cnt_y = h->d_cnt + 4;
    a.bdown = h->d_bdown;
    a.sfb_down = h->d_sfb_down;
    a.bnext = h->d_bnext;
    a.bnext_code = h->d_bnext_code;
    a.trace = h->d_trace;
    a.trace_steps = h->trace_steps;
    a.ylog = h->log_y;
    a.ilog = h->log_idx;
    a.wlog = h->log_w;
    a.log_steps = h->log_steps;
    if (h->d_trace) {
        TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_trace, 0, size_t(h->trace_steps) * kTracePoints * 8, h->stream));
    }
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_acc, 0, 2 * (kMaxExperts + 1) * sizeof(double), h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_barrier, 0, sizeof(unsigned), h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_cnt, 0, 5 * sizeof(unsigned), h->stream));
    const bool prof = h->profile && mode == 1;
    if (prof) {
        TTL_TRY_CUDA(h, cudaEventRecordWithFlags(h->stack_ev[0], h->stream, cudaEventRecordExternal));
    }
    for (int l = begin; l < end; ++l) {
        if (!h->host_layers[size_t(l)].tma) {
            return fail(h, TTL_ERR_STATE, "layer " + std::to_string(l) + " has no tensor maps");
        }
    }
    TTL_TRY_CUDA(h, launch_decode_tc(a, h->sms, h->stream));
    if (prof) {
        TTL_TRY_CUDA(h, cudaEventRecordWithFlags(h->stack_ev[1], h->stream, cudaEventRecordExternal));
        h->stack_profiled = true;
        h->stack_steps = int(tokens) * (end - begin);
    }
    h->launches += 1;
    return TTL_OK;
}

// ---- the decode server (ttl_moe_serve) ----
// A resident launch of the decode kernel in mode 2 answers blocking decode
// calls through the mailbox: no launch, copy or stream synchronisation per
// call.  While it is resident no other kernel can run on the GPU, so it
// leaves after the handle's idle limit without a request, and every other
// use of the handle's stream stops it first.

int check_status(ttl_moe *h);

uint32_t mbox_load(const uint32_t *p) {
    return __atomic_load_n(p, __ATOMIC_ACQUIRE);
}
void mbox_store(uint32_t *p, uint32_t v) {
    __atomic_store_n(p, v, __ATOMIC_RELEASE);
}

// Stops a resident server (it leaves at its next wait for a request) and
// waits for the launch to end.
int stop_server(ttl_moe *h) {
    if (!h->serving) {
        return TTL_OK;
    }
    mbox_store(&h->mbox->stop, 1u);
    const cudaError_t e = cudaStreamSynchronize(h->stream);
    h->serving = false;
    mbox_store(&h->mbox->stop, 0u);
    TTL_TRY_CUDA(h, e);
    return TTL_OK;
}

// Launches the server; request number `base` + 1 is its first step.
int launch_server(ttl_moe *h, uint32_t base) {
    h->mbox_base = base;
    mbox_store(&h->mbox->stop, 0u);
    mbox_store(&h->mbox->alive, 1u);
    const int rc = enqueue_stack(h, 0, int(h->cfg.layers), h->d_srv_x, h->d_y, size_t(1) << 30, 2);
    if (rc) {
        mbox_store(&h->mbox->alive, 0u);
        return rc;
    }
    h->serving = true;
    return TTL_OK;
}

// One blocking decode through the server: x and the layer into the mailbox,
// the request number bumped, then a spin on the answer.  A launch that left
// (idle) before taking the request is replaced by one whose first step is it.
int serve_decode(ttl_moe *h, int layer, const float *x, float *out, int32_t *top4_idx, float *top4_w) {
    for (uint32_t l = 0; l < h->cfg.layers; ++l) {
        if (!h->layers[l].uploaded) {
            return fail(h, TTL_ERR_STATE, "the decode server needs every layer uploaded");
        }
    }
    DecodeMailbox *mb = h->mbox;
    if (!h->serving || mbox_load(&mb->alive) == 0u) {
        const int rc = stop_server(h);  // a launch that left: wait for its end
        if (rc) {
            return rc;
        }
        const int lrc = launch_server(h, h->req);
        if (lrc) {
            return lrc;
        }
    }
    std::memcpy(mb->x, x, kDim * sizeof(float));
    const uint32_t r = ++h->req;
    __atomic_store_n(&mb->reqw, (static_cast<unsigned long long>(r) << 32) | uint32_t(layer), __ATOMIC_RELEASE);
    const auto deadline = Clock::now() + std::chrono::milliseconds(h->timeout_ms);
    // the answer is tagged words carrying r: the top-4, then every row value
    auto tag_of = [](const unsigned long long *p) {
        return uint32_t(__atomic_load_n(p, __ATOMIC_ACQUIRE) >> 32);
    };
    int next = 0;  // rows [0, next) carry r
    int top = 0;   // top-4 words [0, top) carry r
    for (uint32_t spins = 0;; ++spins) {
        while (top < 8 && tag_of(&mb->top[top]) == r) {
            ++top;
        }
        while (next < kDim && tag_of(&mb->y[next]) == r) {
            ++next;
        }
        if (top == 8 && next == kDim) {
            break;
        }
        if (mbox_load(&mb->resp) == r) {  // the step reported a failure
            stop_server(h);
            return check_status(h);
        }
        if (mbox_load(&mb->alive) == 0u) {
            // the launch ended without answering: an error it recorded, or
            // it left idle just before the request came
            const int rc = stop_server(h);
            uint32_t st = 0;
            TTL_TRY_CUDA(h, cudaMemcpy(&st, h->d_status, sizeof(st), cudaMemcpyDeviceToHost));
            if (rc || st) {
                return rc ? rc : check_status(h);
            }
            const int lrc = launch_server(h, r - 1);
            if (lrc) {
                return lrc;
            }
            continue;
        }
        if ((spins & 1023u) == 0u) {
            // a launch that failed is reported at once, not at the deadline
            const cudaError_t q = cudaStreamQuery(h->stream);
            if (q != cudaErrorNotReady && q != cudaSuccess) {
                h->serving = false;
                return fail(h, TTL_ERR_CUDA, std::string("decode server: ") + cudaGetErrorString(q));
            }
            if (Clock::now() > deadline) {
                return fail(h, TTL_ERR_DEVICE, "the decode server did not answer within the handle's timeout");
            }
        }
#if defined(__x86_64__)
        __builtin_ia32_pause();
#endif
    }
    for (int k = 0; k < kDim; ++k) {
        const uint32_t bits = uint32_t(mb->y[k]);
        std::memcpy(out + k, &bits, sizeof(float));
    }
    for (int q = 0; q < 4; ++q) {
        if (top4_idx) {
            top4_idx[q] = int32_t(uint32_t(mb->top[q]));
        }
        if (top4_w) {
            const uint32_t bits = uint32_t(mb->top[4 + q]);
            std::memcpy(top4_w + q, &bits, sizeof(float));
        }
    }
    return TTL_OK;
}

// The graph ttl_moe_decode replays for `layer`: the input row from pinned
// staging, one persistent-kernel step, the output block back.  Captured at
// upload and again whenever launch settings change (trace, step log), so the
// blocking call allocates nothing.
int capture_decode_graph(ttl_moe *h, int layer) {
    if (!stack_path(h) || !h->layers[size_t(layer)].uploaded) {
        return TTL_OK;
    }
    auto old = h->decode_graphs.find(layer);
    if (old != h->decode_graphs.end()) {
        cudaGraphExecDestroy(old->second.first);
        h->decode_graphs.erase(old);
    }
    cudaGraph_t graph = nullptr;
    TTL_TRY_CUDA(h, cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
    const uint64_t launches = h->launches;
    cudaMemcpyAsync(h->d_x, h->pin->x, kDim * sizeof(float), cudaMemcpyHostToDevice, h->stream);
    int rc = enqueue_stack(h, layer, layer + 1, h->d_x, h->d_dblk->y, 1, 0);
    cudaMemcpyAsync(&h->pin->out, h->d_dblk, sizeof(h->pin->out), cudaMemcpyDeviceToHost, h->stream);
    const cudaError_t end = cudaStreamEndCapture(h->stream, &graph);
    h->launches = launches;
    if (rc || end != cudaSuccess) {
        if (graph) {
            cudaGraphDestroy(graph);
        }
        return rc ? rc : fail(h, TTL_ERR_CUDA, std::string("stream capture: ") + cudaGetErrorString(end));
    }
    cudaGraphExec_t exec = nullptr;
    const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    if (inst != cudaSuccess) {
        return fail(h, TTL_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(inst));
    }
    // uploaded now, so the first decode call of the layer does not pay for it
    if (cudaGraphUpload(exec, h->stream) != cudaSuccess) {
        cudaGraphExecDestroy(exec);
        return fail(h, TTL_ERR_CUDA, "graph upload failed");
    }
    h->decode_graphs.emplace(layer, std::make_pair(exec, uint64_t(1)));
    return TTL_OK;
}

// Launch settings changed (profiling events, trace, step log): captured
// forward graphs are dropped (recaptured on their next call) and the decode
// graphs recaptured now.
int refresh_graphs(ttl_moe *h) {
    TTL_TRY_CUDA(h, cudaStreamSynchronize(h->stream));
    for (auto &g : h->graphs) {
        cudaGraphExecDestroy(g.second.exec);
    }
    h->graphs.clear();
    for (int l = 0; l < int(h->cfg.layers); ++l) {
        const int rc = capture_decode_graph(h, l);
        if (rc) {
            return rc;
        }
    }
    return TTL_OK;
}

int enqueue_forward(ttl_moe *h, int begin, int end, const float *x, float *y, size_t tokens) {
    if (stack_path(h) && end > begin) {
        return enqueue_stack(h, begin, end, x, y, tokens, 1);
    }
    for (size_t t = 0; t < tokens; ++t) {
        const float *cur = x + t * kDim;
        float *dst = y + t * kDim;
        for (int l = begin; l < end; ++l) {
            cudaEvent_t *ev = nullptr;
            if (h->profile && t == 0 && h->events.size() >= size_t(4 * (l - begin + 1))) {
                ev = &h->events[size_t(4 * (l - begin))];
                h->profile_layers = l - begin + 1;
            }
            int rc = enqueue_decode_layer(h, l, cur, 1, cur, dst, ev);
            if (rc) {
                return rc;
            }
            cur = dst;
        }
        if (begin == end && x != y) {
            TTL_TRY_CUDA(h, cudaMemcpyAsync(dst, cur, kDim * sizeof(float), cudaMemcpyDeviceToDevice, h->stream));
        }
    }
    return TTL_OK;
}

int check_status(ttl_moe *h) {
    uint32_t status = 0;
    TTL_TRY_CUDA(h, cudaMemcpy(&status, h->d_status, sizeof(status), cudaMemcpyDeviceToHost));
    if (status) {
        cudaMemset(h->d_status, 0, sizeof(uint32_t));
        std::string what;
        if (status & kStatusBadExpert) {
            what += " expert-index-out-of-range";
        }
        if (status & kStatusCapacity) {
            what += " capacity-exceeded";
        }
        if (status & kStatusWaitTimeout) {
            what += " bounded-wait-timeout";
        }
        if (status & kStatusBadShape) {
            what += " bad-shape";
        }
        return fail(h, TTL_ERR_DEVICE, "device status:" + what);
    }
    return TTL_OK;
}

int sync_and_check(ttl_moe *h) {
    const int rc = stream_wait(h);
    return rc ? rc : check_status(h);
}

// Expert-parallel prefill of this rank's own tokens over peer memory
// (prefill_ep.cu has the steps): router, plan, rows written into the
// experts' owners' receive blocks, the expert pipeline on the rows received
// from every rank, rows w * down written back into the tokens' owners'
// blocks, owner combine.  All on the stream: no host round trip, no NCCL;
// every wait on a peer is bounded on the device.
int enqueue_prefill_ep(ttl_moe *h, int layer, const float *x, size_t tokens, float *out) {
    const int W = int(h->cfg.world);
    const int R = int(h->cfg.rank);
    const int P = h->expert_count;
    if (!h->ep.mapped) {
        return fail(h, TTL_ERR_UNSUPPORTED, "expert-parallel prefill needs every rank's receive block mapped");
    }
    const LayerDev L = layer_view(h, layer);
    const TmaDesc *tma = h->host_layers[size_t(layer)].tma;
    if (!tma) {
        return fail(h, TTL_ERR_STATE, "layer " + std::to_string(layer) + " has no tensor maps");
    }
    auto &ep = h->ep;
    const uint32_t tag = ++ep.seq;
    const EpInbox in = ep_inbox_at(ep.inbox, W, ep.cap);
    PrefillWork own = h->pw;
    own.logits = ep.own_logits;
    own.top_idx = ep.own_idx;
    own.top_w = ep.own_w;
    own.seg_count = nullptr;
    PrefillShape so{int(h->cfg.experts), h->expert_begin, h->expert_count, int(tokens), h->sms};
    launch_prefill_router(L, own, so, x, h->stream);
    launch_ep_plan(ep.own_idx, int(tokens), W, P, ep.tok_off, ep.cnt, h->stream);
    TTL_TRY_CUDA(h, cudaMemsetAsync(ep.arrive, 0, 2 * sizeof(unsigned), h->stream));
    launch_ep_send(x, ep.own_idx, ep.own_w, int(tokens), W, R, ep.cap, ep.tok_off, ep.cnt, ep.peers, tag, ep.arrive,
                   h->sms, h->stream);
    launch_ep_wait(in.cnt, W, tag, ep.cap, ep.rcnt, h->d_status, h->stream);
    // this rank's experts on the rows received from every rank
    PrefillShape sp{int(h->cfg.experts), h->expert_begin, h->expert_count, W * ep.cap, h->sms};
    launch_prefill_route(h->pw, sp, h->stream);
    launch_prefill_gateup(L, tma, h->pw, sp, in.x, h->stream);
    launch_prefill_down(L, tma, h->pw, sp, h->stream);
    launch_ep_back(h->pw, in, W, R, P, ep.cap, ep.peers, tag, ep.arrive + 1, h->sms, h->stream);
    launch_ep_wait(in.done, W, tag, ep.cap, nullptr, h->d_status, h->stream);
    launch_ep_combine(ep.own_idx, int(tokens), in.back, out, h->stream);
    h->launches += 11;  // router, plan, send, wait, route, split, gate/up, down, back, wait, combine
    TTL_TRY_CUDA(h, cudaGetLastError());
    return TTL_OK;
}

int enqueue_prefill(ttl_moe *h, int layer, const float *x, size_t tokens, float *out) {
    if (h->cfg.world > 1) {
        return enqueue_prefill_ep(h, layer, x, tokens, out);
    }
    const LayerDev L = layer_view(h, layer);
    PrefillShape s{int(h->cfg.experts), h->expert_begin, h->expert_count, int(tokens), h->sms};
    launch_prefill_router(L, h->pw, s, x, h->stream);
    launch_prefill_route(h->pw, s, h->stream);
    const TmaDesc *tma = h->host_layers[size_t(layer)].tma;
    if (!tma) {
        return fail(h, TTL_ERR_STATE, "layer " + std::to_string(layer) + " has no tensor maps");
    }
    launch_prefill_gateup(L, tma, h->pw, s, x, h->stream);
    launch_prefill_down(L, tma, h->pw, s, h->stream);
    launch_prefill_combine(h->pw, s, out, h->stream);
    h->launches += 6;
    TTL_TRY_CUDA(h, cudaGetLastError());
    return TTL_OK;
}

// The own tokens' top-4 of the last prefill (world > 1: the routing of this
// rank's tokens, not of the tokens it received).
const int32_t *prefill_top_idx(const ttl_moe *h) {
    return h->cfg.world > 1 ? h->ep.own_idx : h->pw.top_idx;
}
const float *prefill_top_w(const ttl_moe *h) {
    return h->cfg.world > 1 ? h->ep.own_w : h->pw.top_w;
}

} // namespace

extern "C" {

int ttl_moe_abi_version(void) {
    return TTL_MOE_ABI_VERSION;
}

const char *ttl_moe_last_error(const ttl_moe *handle) {
    return handle_error(handle);
}

int ttl_moe_nccl_id(void *id_out) {
    if (!id_out) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null id buffer");
    }
    const char *why = nullptr;
    const NcclApi *api = nccl(&why);
    if (!api) {
        return fail(nullptr, TTL_ERR_NCCL, std::string("NCCL unavailable: ") + why);
    }
    ncclUniqueId id;
    const ncclResult_t r = api->GetUniqueId(&id);
    if (r != ncclSuccess) {
        return fail(nullptr, TTL_ERR_NCCL, std::string("ncclGetUniqueId: ") + api->GetErrorString(r));
    }
    static_assert(sizeof(id) == TTL_MOE_NCCL_ID_BYTES, "ncclUniqueId size");
    std::memcpy(id_out, &id, sizeof(id));
    return TTL_OK;
}

int ttl_moe_create(const ttl_moe_config *config, ttl_moe **handle_out) {
    if (!config || !handle_out) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null config or handle pointer");
    }
    *handle_out = nullptr;
    const ttl_moe_config &c = *config;
    if (c.experts != 32 && c.experts != 128) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "experts must be 32 or 128");
    }
    if (c.layers < 1 || c.layers > 36) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "layers must be in 1..36");
    }
    if (c.world != 1 && c.world != 2 && c.world != 4 && c.world != 8) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "world must be 1, 2, 4 or 8");
    }
    if (c.rank >= c.world) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "rank must be below world");
    }
    if (c.world > 1 && !c.nccl_id) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "world > 1 needs an NCCL id");
    }
    if (c.max_tokens > (1u << 16)) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "max_tokens above 65536");
    }
    int count = 0;
    if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
        cudaGetLastError();
        return fail(nullptr, TTL_ERR_UNSUPPORTED, "no CUDA device");
    }
    int device = c.device;
    if (device < 0) {
        if (cudaGetDevice(&device) != cudaSuccess) {
            return fail(nullptr, TTL_ERR_CUDA, "cudaGetDevice failed");
        }
    }
    if (device >= count) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "device ordinal out of range");
    }
    cudaDeviceProp prop{};
    if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) {
        return fail(nullptr, TTL_ERR_CUDA, "cudaGetDeviceProperties failed");
    }
    if (prop.major != 10) {
        return fail(nullptr, TTL_ERR_UNSUPPORTED,
                    "the kernels are built for sm_100a (B200); device is sm_" + std::to_string(prop.major) +
                        std::to_string(prop.minor));
    }

    ttl_moe *h = new ttl_moe();
    h->cfg = c;
    h->cfg.nccl_id = nullptr;
    h->device = device;
    h->sms = prop.multiProcessorCount;
    h->expert_count = int(c.experts / c.world);
    h->expert_begin = int(c.rank) * h->expert_count;
    h->layers.resize(c.layers);
    h->host_layers.resize(c.layers);

    auto bail = [&](int rc) {
        std::string msg = h->error;
        ttl_moe_destroy(h);
        fail(nullptr, rc, msg);
        return rc;
    };
    if (cudaSetDevice(device) != cudaSuccess) {
        return bail(fail(h, TTL_ERR_CUDA, "cudaSetDevice failed"));
    }
    if (cudaStreamCreateWithFlags(&h->stream, cudaStreamNonBlocking) != cudaSuccess) {
        return bail(fail(h, TTL_ERR_CUDA, "cudaStreamCreate failed"));
    }
    configure_decode_kernels();
    configure_prefill_kernels();
    configure_prefill_tc();
    configure_prefill_ep();
    configure_decode_tc();
    if (cudaEventCreate(&h->stack_ev[0]) != cudaSuccess || cudaEventCreate(&h->stack_ev[1]) != cudaSuccess) {
        return bail(fail(h, TTL_ERR_CUDA, "cudaEventCreate failed"));
    }

    const size_t E = c.experts;
    const size_t T = std::max<uint32_t>(c.max_tokens, 1u);
    int rc = TTL_OK;
    rc = rc ? rc : alloc_n(h, &h->d_dblk, 1);
    if (!rc) {
        h->d_status = &h->d_dblk->status;
        h->dw.top_idx = h->d_dblk->idx;
        h->dw.top_w = h->d_dblk->w;
    }
    // host-call staging: the blocking decode's pinned block and the forward
    // call's device rows (ttl_moe_forward works through them in chunks)
    h->fwd_cap = std::max<size_t>(c.max_tokens, kForwardStagingTokens);
    rc = rc ? rc : alloc_n(h, &h->d_fwd, h->fwd_cap * kDim);
    if (!rc && cudaHostAlloc(reinterpret_cast<void **>(&h->pin), sizeof(*h->pin), cudaHostAllocDefault) != cudaSuccess) {
        h->pin = nullptr;
        rc = fail(h, TTL_ERR_CUDA, "cudaHostAlloc of the decode staging failed");
    }
    rc = rc ? rc : alloc_n(h, &h->d_counters, 4);
    rc = rc ? rc : alloc_n(h, &h->d_ones, kDim);
    rc = rc ? rc : alloc_n(h, &h->dw.h, kDim);
    rc = rc ? rc : alloc_n(h, &h->dw.logits, 2 * size_t(kMaxExperts));
    rc = rc ? rc : alloc_n(h, &h->dw.bounds, 2 * size_t(kMaxExperts));
    rc = rc ? rc : alloc_n(h, &h->dw.hidden, 4 * size_t(kDim));
    rc = rc ? rc : alloc_n(h, &h->dw.partial, kDim);
    rc = rc ? rc : alloc_n(h, &h->dw.arrive, 1);
    rc = rc ? rc : alloc_n(h, &h->d_x, T * kDim);
    rc = rc ? rc : alloc_n(h, &h->d_y, T * kDim);
    rc = rc ? rc : alloc_n(h, &h->d_layers, c.layers);
    rc = rc ? rc : alloc_n(h, &h->d_tma, size_t(c.layers) * kTmaCount);
    rc = rc ? rc : alloc_n(h, &h->d_pack_flags, 1);
    rc = rc ? rc : alloc_n(h, &h->d_acc, 2 * (kMaxExperts + 1));
    rc = rc ? rc : alloc_n(h, &h->d_barrier, 2);
    rc = rc ? rc : alloc_n(h, &h->d_part_gu, kPartGuWords);
    rc = rc ? rc : alloc_n(h, &h->d_part_dn, kPartDnWords);
    rc = rc ? rc : alloc_n(h, &h->d_rpt, kRptWords);
    rc = rc ? rc : alloc_n(h, &h->d_rlog, kRlogWords);
    rc = rc ? rc : alloc_n(h, &h->d_cnt, 5);
    rc = rc ? rc : alloc_n(h, &h->d_seq, 2);
    rc = rc ? rc : alloc_n(h, &h->d_bdown, kBdownBytes);
    rc = rc ? rc : alloc_n(h, &h->d_sfb_down, kSfbDownBytes);
    rc = rc ? rc : alloc_n(h, &h->d_bnext, kBnextBytes);
    rc = rc ? rc : alloc_n(h, &h->d_bnext_code, kBnextCodeBytes);
    if (rc) {
        return bail(rc);
    }
    h->dw.counters = h->d_counters;
    h->dw.status = h->d_status;
    if (c.max_tokens > 0) {
        // at world > 1 the expert pipeline runs on the tokens received from
        // every rank (each sends each own token at most once)
        const size_t Tp = size_t(c.world) * T;
        if (c.world > 1) {
            const size_t W = c.world;
            rc = rc ? rc : alloc_n(h, &h->ep.own_idx, 4 * T);
            rc = rc ? rc : alloc_n(h, &h->ep.own_w, 4 * T);
            rc = rc ? rc : alloc_n(h, &h->ep.own_logits, T * E);
            rc = rc ? rc : alloc_n(h, &h->ep.tok_off, T * W);
            rc = rc ? rc : alloc_n(h, &h->ep.cnt, W);
            rc = rc ? rc : alloc_n(h, &h->ep.rcnt, W);
            rc = rc ? rc : alloc_n(h, &h->ep.arrive, 2);
            h->ep.cap = int(T);
            rc = rc ? rc : alloc(h, &h->ep.inbox, ep_inbox_bytes(int(W), int(T)));
            if (!rc && cudaMemset(h->ep.inbox, 0, ep_inbox_bytes(int(W), int(T))) != cudaSuccess) {
                rc = fail(h, TTL_ERR_CUDA, "cannot clear the receive block");
            }
        }
        const size_t pairs = 4 * Tp;
        rc = rc ? rc : alloc_n(h, &h->pw.logits, Tp * E);
        rc = rc ? rc : alloc_n(h, &h->pw.top_idx, pairs);
        rc = rc ? rc : alloc_n(h, &h->pw.top_w, pairs);
        rc = rc ? rc : alloc_n(h, &h->pw.counts, E);
        rc = rc ? rc : alloc_n(h, &h->pw.offsets, E + 1);
        // slots: each local expert's pairs padded to 16
        const size_t groups = prefill_groups(Tp, size_t(h->expert_count));
        const size_t slots = 16 * groups;
        rc = rc ? rc : alloc_n(h, &h->pw.pair_token, slots);
        rc = rc ? rc : alloc_n(h, &h->pw.pair_slot, pairs);
        rc = rc ? rc : alloc_n(h, &h->pw.tiles, groups);
        rc = rc ? rc : alloc_n(h, &h->pw.tile_count, 1);
        rc = rc ? rc : alloc_n(h, &h->pw.units, groups);
        rc = rc ? rc : alloc_n(h, &h->pw.unit_count, 1);
        rc = rc ? rc : alloc_n(h, &h->pw.down, slots * kDim);
        const size_t units = prefill_units(Tp, size_t(h->expert_count));
        rc = rc ? rc : alloc_n(h, &h->pw.bdig, units * kPrefillUnitBytes);
        rc = rc ? rc : alloc_n(h, &h->pw.bsfb, units * kPrefillUnitScaleBytes);
        rc = rc ? rc : alloc_n(h, &h->pw.bdig_dn, units * kPrefillUnitBytes);
        rc = rc ? rc : alloc_n(h, &h->pw.bsfb_dn, units * kPrefillUnitScaleBytes);
        h->pw.status = h->d_status;
        if (!rc && c.world > 1) {
            // the expert pipeline runs on the received rows: [world][T] by
            // source rank, the ids and weights sent with them
            const EpInbox in = ep_inbox_at(h->ep.inbox, int(c.world), int(T));
            h->pw.top_idx = in.idx;
            h->pw.top_w = in.w;
            h->pw.seg_count = h->ep.rcnt;
            h->pw.seg_rows = int(T);
        }
        if (rc) {
            return bail(rc);
        }
    }
    std::vector<float> ones(kDim, 1.0f);
    if (cudaMemcpy(h->d_ones, ones.data(), kDim * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemset(h->d_status, 0, sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(h->d_counters, 0, 4 * sizeof(unsigned long long)) != cudaSuccess ||
        cudaMemset(h->dw.arrive, 0, sizeof(unsigned int)) != cudaSuccess ||
        cudaMemset(h->dw.top_idx, 0, 4 * sizeof(int32_t)) != cudaSuccess ||
        cudaMemset(h->dw.top_w, 0, 4 * sizeof(float)) != cudaSuccess ||
        cudaMemset(h->d_barrier, 0, 2 * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(h->d_cnt, 0, 5 * sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(h->d_seq, 0, 2 * sizeof(uint32_t)) != cudaSuccess ||
        cudaMemset(h->d_part_gu, 0, kPartGuWords * 8) != cudaSuccess ||
        cudaMemset(h->d_part_dn, 0, kPartDnWords * 8) != cudaSuccess ||
        cudaMemset(h->d_rpt, 0, kRptWords * 8) != cudaSuccess ||
        cudaMemset(h->d_rlog, 0, kRlogWords * 8) != cudaSuccess ||
        cudaMemset(h->d_bdown, 0, kBdownBytes) != cudaSuccess ||
        cudaMemset(h->d_sfb_down, 0x7f, kSfbDownBytes) != cudaSuccess ||
        cudaMemset(h->d_bnext, 0, kBnextBytes) != cudaSuccess ||
        cudaMemset(h->d_bnext_code, 0x7f, kBnextCodeBytes) != cudaSuccess ||
        cudaMemset(h->d_layers, 0, c.layers * sizeof(StackLayer)) != cudaSuccess) {
        return bail(fail(h, TTL_ERR_CUDA, "device initialisation failed"));
    }
    if (c.world > 1) {
        const char *why = nullptr;
        const NcclApi *api = nccl(&why);
        if (!api) {
            return bail(fail(h, TTL_ERR_NCCL, std::string("NCCL unavailable: ") + why));
        }
        if (alloc_n(h, &h->d_sync, 4) != TTL_OK ||
            cudaEventCreateWithFlags(&h->wait_ev, cudaEventDisableTiming) != cudaSuccess) {
            return bail(fail(h, TTL_ERR_CUDA, "cannot allocate the resync scratch"));
        }
        ncclUniqueId id;
        std::memcpy(&id, c.nccl_id, sizeof(id));
        ncclConfig_t nc = NCCL_CONFIG_INITIALIZER;
        nc.blocking = 0;  // every wait on the communicator is bounded on the host
        const ncclResult_t r = api->CommInitRankConfig(&h->comm, int(c.world), id, int(c.rank), &nc);
        if (r != ncclSuccess && r != ncclInProgress) {
            h->comm = nullptr;
            return bail(fail(h, TTL_ERR_NCCL, std::string("ncclCommInitRankConfig: ") + api->GetErrorString(r)));
        }
        int xrc = comm_settle(h, "ncclCommInitRankConfig");
        xrc = xrc ? xrc : setup_exchange(h);
        if (xrc) {
            return bail(xrc);
        }
    }
    *handle_out = h;
    return TTL_OK;
}

void ttl_moe_destroy(ttl_moe *h) {
    if (!h) {
        return;
    }
    cudaSetDevice(h->device);
    stop_server(h);
    if (h->stream) {
        stream_wait(h);  // bounded for a multi-rank handle
    }
    if (h->mbox) {
        cudaFreeHost(h->mbox);
    }
    for (auto &g : h->graphs) {
        cudaGraphExecDestroy(g.second.exec);
    }
    h->graphs.clear();
    for (auto &g : h->decode_graphs) {
        cudaGraphExecDestroy(g.second.first);
    }
    h->decode_graphs.clear();
    if (h->pin) {
        cudaFreeHost(h->pin);
    }
    for (cudaEvent_t e : h->events) {
        cudaEventDestroy(e);
    }
    for (cudaEvent_t e : h->stack_ev) {
        if (e) {
            cudaEventDestroy(e);
        }
    }
    for (void *p : h->xch_open) {
        if (p) {
            cudaIpcCloseMemHandle(p);
        }
    }
    for (void *p : h->ep.open) {
        if (p) {
            cudaIpcCloseMemHandle(p);
        }
    }
    if (h->comm) {
        // finalize (flushes this rank's NCCL work), bounded; abort past the deadline
        const NcclApi *api = nccl(nullptr);
        const ncclResult_t f = api->CommFinalize(h->comm);
        if ((f == ncclSuccess || f == ncclInProgress) && comm_settle(h, "ncclCommFinalize") == TTL_OK) {
            api->CommDestroy(h->comm);
        } else if (h->comm) {
            api->CommAbort(h->comm);
        }
        h->comm = nullptr;
    }
    if (h->wait_ev) {
        cudaEventDestroy(h->wait_ev);
    }
    for (void *p : h->allocations) {
        cudaFree(p);
    }
    if (h->stream) {
        cudaStreamDestroy(h->stream);
    }
    delete h;
}

} // extern "C"

namespace {

// Both uploads: GGUF blocks are packed on the device; packed payloads
// (TTL_TTQ_FORMAT_MXFP4_GPU) are copied and only their scales checked.
int upload_layer(ttl_moe *h, int layer, const float *router_w, const float *router_b, const void *gate_w,
                 const float *gate_b, const void *up_w, const float *up_b, const void *down_w, const float *down_b,
                 bool packed) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (layer < 0 || layer >= int(h->cfg.layers)) {
        return fail(h, TTL_ERR_ARGUMENT, "layer out of range");
    }
    if (!router_w || !router_b || !gate_w || !gate_b || !up_w || !up_b || !down_w || !down_b) {
        return fail(h, TTL_ERR_ARGUMENT, "null tensor pointer");
    }
    int rc = set_device(h);
    if (rc) {
        return rc;
    }
    LayerStore &s = h->layers[size_t(layer)];
    const size_t E = h->cfg.experts;
    const size_t El = size_t(h->expert_count);
    if (!s.router_w) {
        rc = rc ? rc : alloc_n(h, &s.router_w, E * kDim);
        rc = rc ? rc : alloc_n(h, &s.router_b, E);
        rc = rc ? rc : alloc_n(h, &s.gate, El * kPackedMatrixBytes);
        rc = rc ? rc : alloc_n(h, &s.up, El * kPackedMatrixBytes);
        rc = rc ? rc : alloc_n(h, &s.down, El * kPackedMatrixBytes);
        rc = rc ? rc : alloc_n(h, &s.gate_b, El * kDim);
        rc = rc ? rc : alloc_n(h, &s.up_b, El * kDim);
        rc = rc ? rc : alloc_n(h, &s.down_b, El * kDim);
        if (rc) {
            return rc;
        }
    }
    const size_t expert_gguf = packed ? kPackedMatrixBytes : size_t(kDim) * kGgufRowBytes;
    const size_t first = size_t(h->expert_begin);
    TTL_TRY_CUDA(h, cudaMemcpy(s.router_w, router_w, E * kDim * sizeof(float), cudaMemcpyDefault));
    TTL_TRY_CUDA(h, cudaMemcpy(s.router_b, router_b, E * sizeof(float), cudaMemcpyDefault));
    TTL_TRY_CUDA(h, cudaMemcpy(s.gate_b, gate_b + first * kDim, El * kDim * sizeof(float), cudaMemcpyDefault));
    TTL_TRY_CUDA(h, cudaMemcpy(s.up_b, up_b + first * kDim, El * kDim * sizeof(float), cudaMemcpyDefault));
    TTL_TRY_CUDA(h, cudaMemcpy(s.down_b, down_b + first * kDim, El * kDim * sizeof(float), cudaMemcpyDefault));
    const void *srcs[3] = {gate_w, up_w, down_w};
    uint8_t *dsts[3] = {s.gate, s.up, s.down};
    for (int m = 0; m < 3; ++m) {
        const uint8_t *src = (const uint8_t *)srcs[m] + first * expert_gguf;
        if (!is_device_pointer(srcs[m])) {
            if (!h->staging) {
                // sized for either input layout, so GGUF and packed uploads can be mixed on one handle
                h->staging_bytes = El * std::max(kPackedMatrixBytes, size_t(kDim) * kGgufRowBytes);
                rc = alloc(h, reinterpret_cast<void **>(&h->staging), h->staging_bytes);
                if (rc) {
                    return rc;
                }
            }
            TTL_TRY_CUDA(h, cudaMemcpy(h->staging, src, El * expert_gguf, cudaMemcpyHostToDevice));
            src = h->staging;
        }
        TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_pack_flags, 0, sizeof(uint32_t), h->stream));
        if (packed) {
            TTL_TRY_CUDA(h, cudaMemcpyAsync(dsts[m], src, El * kPackedMatrixBytes, cudaMemcpyDefault, h->stream));
            launch_scan_scales(dsts[m], El, h->stream, h->d_pack_flags);
        } else {
            launch_pack(src, dsts[m], El, h->stream, h->d_pack_flags);
        }
        TTL_TRY_CUDA(h, cudaGetLastError());
        uint32_t flags = 0;
        TTL_TRY_CUDA(h, cudaMemcpyAsync(&flags, h->d_pack_flags, sizeof(flags), cudaMemcpyDeviceToHost, h->stream));
        TTL_TRY_CUDA(h, cudaStreamSynchronize(h->stream));
        if (flags & 1u) {
            return fail(h, TTL_ERR_UNSUPPORTED,
                        "layer " + std::to_string(layer) +
                            ": an MXFP4 scale byte is 255 (2^128 in tt-lab's convention), which the tensor cores' "
                            "E8M0 scales cannot represent");
        }
    }
    s.uploaded = true;
    const int prc = push_layer_descriptor(h, layer);
    return prc ? prc : capture_decode_graph(h, layer);
}

} // namespace

extern "C" {

int ttl_moe_upload_layer(ttl_moe *h, int layer, const float *router_w, const float *router_b, const void *gate_w,
                         const float *gate_b, const void *up_w, const float *up_b, const void *down_w,
                         const float *down_b) {
    return upload_layer(h, layer, router_w, router_b, gate_w, gate_b, up_w, up_b, down_w, down_b, false);
}

int ttl_moe_upload_layer_packed(ttl_moe *h, int layer, const float *router_w, const float *router_b,
                                const void *gate_packed, const float *gate_b, const void *up_packed, const float *up_b,
                                const void *down_packed, const float *down_b) {
    return upload_layer(h, layer, router_w, router_b, gate_packed, gate_b, up_packed, up_b, down_packed, down_b, true);
}



int ttl_moe_upload_norm(ttl_moe *h, int layer, const float *norm_w) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (layer < 0 || layer >= int(h->cfg.layers) || !norm_w) {
        return fail(h, TTL_ERR_ARGUMENT, "bad layer or null weights");
    }
    int rc = set_device(h);
    LayerStore &s = h->layers[size_t(layer)];
    if (!s.norm_w) {
        rc = rc ? rc : alloc_n(h, &s.norm_w, kDim);
    }
    if (rc) {
        return rc;
    }
    TTL_TRY_CUDA(h, cudaMemcpy(s.norm_w, norm_w, kDim * sizeof(float), cudaMemcpyDefault));
    return push_layer_descriptor(h, layer);
}

int ttl_moe_decode_async(ttl_moe *h, int layer, const float *x, float *out, int32_t *top4_idx, float *top4_w) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (const int frc = ep_ready(h)) {
        return frc;
    }
    if (!x || !out) {
        return fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    int rc = check_layer(h, layer);
    rc = rc ? rc : set_device(h);
    if (!rc && stack_path(h)) {
        rc = enqueue_stack(h, layer, layer + 1, x, out, 1, 0);
    } else if (!rc) {
        rc = enqueue_decode_layer(h, layer, x, 0, nullptr, out);
    }
    if (rc) {
        return rc;
    }
    if (top4_idx) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_idx, h->dw.top_idx, 4 * sizeof(int32_t), cudaMemcpyDeviceToDevice,
                                        h->stream));
    }
    if (top4_w) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_w, h->dw.top_w, 4 * sizeof(float), cudaMemcpyDeviceToDevice,
                                        h->stream));
    }
    return TTL_OK;
}

int ttl_moe_decode(ttl_moe *h, int layer, const float *x, float *out, int32_t *top4_idx, float *top4_w) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int frc = ep_ready(h)) {
        return frc;
    }
    if (!x || !out) {
        return fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    int rc = check_layer(h, layer);
    rc = rc ? rc : set_device(h);
    if (rc) {
        return rc;
    }
    if (h->serve_idle_us) {
        return serve_decode(h, layer, x, out, top4_idx, top4_w);
    }
    if (!stack_path(h)) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(h->d_x, x, kDim * sizeof(float), cudaMemcpyHostToDevice, h->stream));
        rc = stack_path(h) ? enqueue_stack(h, layer, layer + 1, h->d_x, h->d_y, 1, 0)
                           : enqueue_decode_layer(h, layer, h->d_x, 0, nullptr, h->d_y);
        if (rc) {
            return rc;
        }
        TTL_TRY_CUDA(h, cudaMemcpyAsync(out, h->d_y, kDim * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
        if (top4_idx) {
            TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_idx, h->dw.top_idx, 4 * sizeof(int32_t), cudaMemcpyDeviceToHost,
                                            h->stream));
        }
        if (top4_w) {
            TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_w, h->dw.top_w, 4 * sizeof(float), cudaMemcpyDeviceToHost,
                                            h->stream));
        }
        return sync_and_check(h);
    }
    // one launch of the layer's graph (captured at upload): the input from
    // pinned staging, the persistent kernel, one copy of the output block
    // (output, top-4, status word) back to it
    auto found = h->decode_graphs.find(layer);
    if (found == h->decode_graphs.end()) {
        return fail(h, TTL_ERR_STATE, "layer " + std::to_string(layer) + " has no decode graph");
    }
    std::memcpy(h->pin->x, x, kDim * sizeof(float));
    TTL_TRY_CUDA(h, cudaGraphLaunch(found->second.first, h->stream));
    h->launches += found->second.second;
    rc = stream_wait(h);
    if (rc) {
        return rc;
    }
    if (h->pin->out.status) {
        return check_status(h);  // reads, clears and reports the device status word
    }
    std::memcpy(out, h->pin->out.y, kDim * sizeof(float));
    if (top4_idx) {
        std::memcpy(top4_idx, h->pin->out.idx, 4 * sizeof(int32_t));
    }
    if (top4_w) {
        std::memcpy(top4_w, h->pin->out.w, 4 * sizeof(float));
    }
    return TTL_OK;
}

int ttl_moe_prefill_async(ttl_moe *h, int layer, const float *x, size_t tokens, float *out, int32_t *top4_idx,
                          float *top4_w) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (const int frc = ep_ready(h)) {
        return frc;
    }
    if (!x || !out) {
        return fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    if (reinterpret_cast<uintptr_t>(x) % 16 != 0) {
        return fail(h, TTL_ERR_ARGUMENT, "prefill input must be 16-byte aligned");
    }
    if (tokens == 0) {
        return fail(h, TTL_ERR_ARGUMENT, "prefill needs at least one token");  // src/model.cpp:464-466
    }
    if (tokens > h->cfg.max_tokens) {
        return fail(h, TTL_ERR_STATE, "prefill exceeds startup batch capacity");  // src/model.cpp:470-472
    }
    int rc = check_layer(h, layer);
    rc = rc ? rc : set_device(h);
    rc = rc ? rc : enqueue_prefill(h, layer, x, tokens, out);
    if (rc) {
        return rc;
    }
    if (top4_idx) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_idx, prefill_top_idx(h), tokens * 4 * sizeof(int32_t),
                                        cudaMemcpyDeviceToDevice, h->stream));
    }
    if (top4_w) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_w, prefill_top_w(h), tokens * 4 * sizeof(float), cudaMemcpyDeviceToDevice,
                                        h->stream));
    }
    return TTL_OK;
}

int ttl_moe_prefill(ttl_moe *h, int layer, const float *x, size_t tokens, float *out, int32_t *top4_idx,
                    float *top4_w) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (const int frc = ep_ready(h)) {
        return frc;
    }
    if (!x || !out) {
        return fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    if (tokens == 0) {
        return fail(h, TTL_ERR_ARGUMENT, "prefill needs at least one token");
    }
    if (tokens > h->cfg.max_tokens) {
        return fail(h, TTL_ERR_STATE, "prefill exceeds startup batch capacity");
    }
    int rc = check_layer(h, layer);
    rc = rc ? rc : set_device(h);
    if (rc) {
        return rc;
    }
    TTL_TRY_CUDA(h, cudaMemcpyAsync(h->d_x, x, tokens * kDim * sizeof(float), cudaMemcpyHostToDevice, h->stream));
    rc = enqueue_prefill(h, layer, h->d_x, tokens, h->d_y);
    if (rc) {
        return rc;
    }
    TTL_TRY_CUDA(h, cudaMemcpyAsync(out, h->d_y, tokens * kDim * sizeof(float), cudaMemcpyDeviceToHost, h->stream));
    if (top4_idx) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_idx, prefill_top_idx(h), tokens * 4 * sizeof(int32_t),
                                        cudaMemcpyDeviceToHost, h->stream));
    }
    if (top4_w) {
        TTL_TRY_CUDA(h, cudaMemcpyAsync(top4_w, prefill_top_w(h), tokens * 4 * sizeof(float), cudaMemcpyDeviceToHost,
                                        h->stream));
    }
    return sync_and_check(h);
}

int ttl_moe_forward_async(ttl_moe *h, int layer_begin, int layer_end, const float *x, float *y, size_t tokens) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (const int frc = ep_ready(h)) {
        return frc;
    }
    if (!x || !y) {
        return fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    if (layer_begin < 0 || layer_end < layer_begin || layer_end > int(h->cfg.layers)) {
        return fail(h, TTL_ERR_ARGUMENT, "bad layer range");
    }
    int rc = set_device(h);
    for (int l = layer_begin; l < layer_end && !rc; ++l) {
        rc = check_layer(h, l);
    }
    if (rc || tokens == 0) {
        return rc;
    }
    // The token loop is captured once per (buffers, count, layers) and
    // replayed; the cache keeps the kMaxForwardGraphs most recently used.
    const GraphKey key{x, y, tokens, layer_begin, layer_end};
    auto found = h->graphs.find(key);
    if (found == h->graphs.end()) {
        if (h->graphs.size() >= kMaxForwardGraphs) {
            auto oldest = h->graphs.begin();
            for (auto it = h->graphs.begin(); it != h->graphs.end(); ++it) {
                if (it->second.last_use < oldest->second.last_use) {
                    oldest = it;
                }
            }
            cudaGraphExecDestroy(oldest->second.exec);
            h->graphs.erase(oldest);
        }
        cudaGraph_t graph = nullptr;
        TTL_TRY_CUDA(h, cudaStreamBeginCapture(h->stream, cudaStreamCaptureModeThreadLocal));
        const uint64_t launches = h->launches;
        rc = enqueue_forward(h, layer_begin, layer_end, x, y, tokens);
        const cudaError_t end = cudaStreamEndCapture(h->stream, &graph);
        if (rc) {
            if (graph) {
                cudaGraphDestroy(graph);
            }
            return rc;
        }
        if (end != cudaSuccess) {
            return fail(h, TTL_ERR_CUDA, std::string("stream capture: ") + cudaGetErrorString(end));
        }
        cudaGraphExec_t exec = nullptr;
        const cudaError_t inst = cudaGraphInstantiate(&exec, graph, 0);
        cudaGraphDestroy(graph);
        if (inst != cudaSuccess) {
            return fail(h, TTL_ERR_CUDA, std::string("graph instantiate: ") + cudaGetErrorString(inst));
        }
        if (cudaGraphUpload(exec, h->stream) != cudaSuccess) {
            cudaGraphExecDestroy(exec);
            return fail(h, TTL_ERR_CUDA, "graph upload failed");
        }
        const uint64_t per_replay = h->launches - launches;
        h->launches = launches;  // counted per replay below
        found = h->graphs.emplace(key, ttl_moe::ForwardGraph{exec, per_replay, 0}).first;
    }
    found->second.last_use = ++h->graph_clock;
    TTL_TRY_CUDA(h, cudaGraphLaunch(found->second.exec, h->stream));
    h->launches += found->second.kernels;
    return TTL_OK;
}

int ttl_moe_forward(ttl_moe *h, int layer_begin, int layer_end, const float *x, float *y, size_t tokens) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int frc = ep_ready(h)) {
        return frc;
    }
    if (!x || !y) {
        return fail(h, TTL_ERR_ARGUMENT, "null input or output");
    }
    int rc = set_device(h);
    if (rc || tokens == 0) {
        return rc;
    }
    // the tokens are independent, so they go through the staging rows (made
    // at create) in chunks of its capacity
    for (size_t t0 = 0; t0 < tokens; t0 += h->fwd_cap) {
        const size_t n = std::min(h->fwd_cap, tokens - t0);
        TTL_TRY_CUDA(h, cudaMemcpyAsync(h->d_fwd, x + t0 * kDim, n * kDim * sizeof(float), cudaMemcpyHostToDevice,
                                        h->stream));
        rc = ttl_moe_forward_async(h, layer_begin, layer_end, h->d_fwd, h->d_fwd, n);
        if (rc) {
            return rc;
        }
        TTL_TRY_CUDA(h, cudaMemcpyAsync(y + t0 * kDim, h->d_fwd, n * kDim * sizeof(float), cudaMemcpyDeviceToHost,
                                        h->stream));
    }
    return sync_and_check(h);
}

int ttl_moe_profile(ttl_moe *h, int enable) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    int rc = set_device(h);
    if (rc) {
        return rc;
    }
    if (enable && h->events.empty()) {
        h->events.resize(size_t(4) * h->cfg.layers);
        for (cudaEvent_t &e : h->events) {
            TTL_TRY_CUDA(h, cudaEventCreate(&e));
        }
    }
    if (h->profile != (enable != 0)) {
        h->profile = enable != 0;
        return refresh_graphs(h);
    }
    return TTL_OK;
}

int ttl_moe_trace(ttl_moe *h, int steps, uint64_t *out) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    int rc = set_device(h);
    if (rc) {
        return rc;
    }
    if (steps > 0 && !h->d_trace) {
        rc = alloc_n(h, &h->d_trace, size_t(steps) * kTracePoints);
        if (rc) {
            return rc;
        }
        h->trace_steps = steps;
        rc = refresh_graphs(h);
        if (rc) {
            return rc;
        }
    }
    if (out && h->d_trace) {
        TTL_TRY_CUDA(h, cudaStreamSynchronize(h->stream));
        TTL_TRY_CUDA(h, cudaMemcpy(out, h->d_trace, size_t(h->trace_steps) * kTracePoints * 8, cudaMemcpyDeviceToHost));
    }
    return TTL_OK;
}

int ttl_moe_record(ttl_moe *h, size_t steps, float *y_log, int32_t *idx_log, float *w_log) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    if (steps > 0 && (!y_log || !idx_log || !w_log)) {
        return fail(h, TTL_ERR_ARGUMENT, "step log needs its three buffers");
    }
    if (steps > size_t(1) << 30) {
        return fail(h, TTL_ERR_ARGUMENT, "step log too long");
    }
    for (const void *p : {(const void *)y_log, (const void *)idx_log, (const void *)w_log}) {
        if (steps > 0 && !is_device_pointer(p)) {
            return fail(h, TTL_ERR_ARGUMENT, "step log buffers must be device memory");
        }
    }
    int rc = set_device(h);
    if (rc) {
        return rc;
    }
    h->log_steps = int(steps);
    h->log_y = steps ? y_log : nullptr;
    h->log_idx = steps ? idx_log : nullptr;
    h->log_w = steps ? w_log : nullptr;
    return refresh_graphs(h);
}

int ttl_moe_kernel_ms(ttl_moe *h, float *ms, size_t n) {
    if (!h || !ms) {
        return fail(h, TTL_ERR_ARGUMENT, "null argument");
    }
    float out[3] = {0.0f, 0.0f, 0.0f};
    if (h->stack_profiled) {
        TTL_TRY_CUDA(h, cudaEventElapsedTime(&out[0], h->stack_ev[0], h->stack_ev[1]));
        out[1] = float(h->stack_steps);
        out[2] = 1.0f;
    } else if (h->profile_layers > 0) {
        double sum = 0.0;
        for (int l = 0; l < h->profile_layers; ++l) {
            float v = 0.0f;
            TTL_TRY_CUDA(h, cudaEventElapsedTime(&v, h->events[size_t(4 * l + 1)], h->events[size_t(4 * l + 2)]));
            sum += v;
        }
        out[0] = float(sum / h->profile_layers);
        out[1] = 1.0f;
        out[2] = 0.0f;
    } else {
        return fail(h, TTL_ERR_STATE, "no profiled forward graph has run");
    }
    for (size_t k = 0; k < n && k < 3; ++k) {
        ms[k] = out[k];
    }
    return TTL_OK;
}

int ttl_moe_sync(ttl_moe *h) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    int rc = set_device(h);
    return rc ? rc : sync_and_check(h);
}

int ttl_moe_serve(ttl_moe *h, uint32_t idle_us) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (idle_us > 1000000u) {
        return fail(h, TTL_ERR_ARGUMENT, "the idle limit is at most 1000000 us");
    }
    if (idle_us && h->cfg.world != 1) {
        return fail(h, TTL_ERR_UNSUPPORTED, "the decode server runs on single-GPU handles");
    }
    int rc = set_device(h);
    rc = rc ? rc : stop_server(h);
    if (rc) {
        return rc;
    }
    if (idle_us && !h->mbox) {
        void *p = nullptr;
        if (cudaHostAlloc(&p, sizeof(DecodeMailbox), cudaHostAllocMapped) != cudaSuccess) {
            cudaGetLastError();
            return fail(h, TTL_ERR_CUDA, "cannot allocate the decode server's mailbox");
        }
        std::memset(p, 0, sizeof(DecodeMailbox));
        h->mbox = static_cast<DecodeMailbox *>(p);
        void *dev = nullptr;
        TTL_TRY_CUDA(h, cudaHostGetDevicePointer(&dev, p, 0));
        h->mbox_dev = static_cast<DecodeMailbox *>(dev);
        rc = alloc_n(h, &h->d_srv_x, kDim);
        rc = rc ? rc : alloc_n(h, &h->d_go, 1);
        if (rc) {
            return rc;
        }
        TTL_TRY_CUDA(h, cudaMemset(h->d_go, 0, sizeof(unsigned long long)));
    }
    h->serve_idle_us = idle_us;
    return TTL_OK;
}

int ttl_moe_set_timeout(ttl_moe *h, uint32_t ms) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (ms == 0) {
        return fail(h, TTL_ERR_ARGUMENT, "timeout must be at least 1 ms");
    }
    h->timeout_ms = ms;
    return TTL_OK;
}

// Collective over the ranks of a multi-rank handle, after a failed call on
// any of them: (1) drain this rank's stream; (2) NCCL max of the ranks' tag
// bases (the persistent kernel's, on the device, and the prefill call tag) --
// a barrier, so every rank's kernels have ended when it returns; (3) this
// rank's exchange buffer, receive-block flags, tagged partials and status
// cleared and the agreed bases installed; (4) a second barrier, so no rank
// launches (and writes into a peer's memory) before every rank has cleared
// its own.  Stale words of a failed launch cannot then match a new tag.
int ttl_moe_resync(ttl_moe *h) {
    if (!h) {
        return fail(nullptr, TTL_ERR_ARGUMENT, "null handle");
    }
    if (const int src = stop_server(h)) {  // a resident decode server leaves the stream first
        return src;
    }
    int rc = set_device(h);
    if (rc) {
        return rc;
    }
    if (h->cfg.world == 1) {
        rc = stream_wait(h);
        TTL_TRY_CUDA(h, cudaMemset(h->d_status, 0, sizeof(uint32_t)));
        return rc;
    }
    if (h->comm_dead) {
        return fail(h, TTL_ERR_NCCL, "the communicator was aborted after a failure; destroy the handle");
    }
    const NcclApi *api = nccl(nullptr);
    rc = stream_wait(h);
    if (rc) {
        return rc;
    }
    TTL_TRY_CUDA(h, cudaMemcpyAsync(h->d_sync, h->d_seq, sizeof(uint32_t), cudaMemcpyDeviceToDevice, h->stream));
    TTL_TRY_CUDA(h, cudaMemcpyAsync(h->d_sync + 1, &h->ep.seq, sizeof(uint32_t), cudaMemcpyHostToDevice, h->stream));
    rc = nccl_check(h, api->AllReduce(h->d_sync, h->d_sync, 2, ncclUint32, ncclMax, h->comm, h->stream),
                    "ncclAllReduce (resync)");
    rc = rc ? rc : stream_wait(h);
    if (rc) {
        return rc;
    }
    uint32_t agreed[2] = {0, 0};
    TTL_TRY_CUDA(h, cudaMemcpy(agreed, h->d_sync, sizeof(agreed), cudaMemcpyDeviceToHost));
    h->ep.seq = agreed[1];
    TTL_TRY_CUDA(h, cudaMemcpyAsync(h->d_seq, h->d_sync, sizeof(uint32_t), cudaMemcpyDeviceToDevice, h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_seq + 1, 0, sizeof(uint32_t), h->stream));
    if (h->d_xch) {
        TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_xch, 0, xch_words(int(h->cfg.world)) * sizeof(unsigned long long),
                                        h->stream));
    }
    if (h->ep.inbox) {
        const EpInbox in = ep_inbox_at(h->ep.inbox, int(h->cfg.world), h->ep.cap);
        TTL_TRY_CUDA(h, cudaMemsetAsync(in.cnt, 0, h->cfg.world * sizeof(unsigned long long), h->stream));
        TTL_TRY_CUDA(h, cudaMemsetAsync(in.done, 0, h->cfg.world * sizeof(unsigned long long), h->stream));
    }
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_part_gu, 0, kPartGuWords * 8, h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_part_dn, 0, kPartDnWords * 8, h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_rpt, 0, kRptWords * 8, h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_rlog, 0, kRlogWords * 8, h->stream));
    TTL_TRY_CUDA(h, cudaMemsetAsync(h->d_status, 0, sizeof(uint32_t), h->stream));
    rc = nccl_check(h, api->AllReduce(h->d_sync, h->d_sync + 2, 1, ncclUint32, ncclMax, h->comm, h->stream),
                    "ncclAllReduce (resync barrier)");
    rc = rc ? rc : stream_wait(h);
    if (rc) {
        return rc;
    }
    h->ep_fault = false;
    return TTL_OK;
}

void *ttl_moe_stream(ttl_moe *h) {
    return h ? (void *)h->stream : nullptr;
}

int ttl_moe_counters(const ttl_moe *h, uint64_t *out, size_t n) {
    if (!h || !out) {
        return 0;
    }
    unsigned long long dev[4] = {0, 0, 0, 0};
    cudaSetDevice(h->device);
    cudaMemcpy(dev, h->d_counters, sizeof(dev), cudaMemcpyDeviceToHost);
    const uint64_t vals[4] = {dev[0], dev[1], h->launches, stack_path(h) ? 1u : 0u};
    const size_t k = std::min<size_t>(n, 4);
    for (size_t i = 0; i < k; ++i) {
        out[i] = vals[i];
    }
    return int(k);
}

} // extern "C"
