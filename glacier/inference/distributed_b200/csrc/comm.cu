// comm.cu -- multi-GPU plumbing of the C ABI for hosts without torch.distributed
// (the reference's C# host over P/Invoke): an NCCL communicator, the pipeline
// stage boundary and the all-to-all exchanges of the expert-parallel layer.
//
// Replaces the reference's LAN transport at a stage boundary -- activations
// quantised with QuantizationKernels.QuantizeBatch (Protocol/
// QuantizationKernels.cs:134-146), framed with a FusedActivationHeader
// (Protocol/FusedActivationHeader.cs:41-125) and written to a socket
// (FusedSocketTransport.cs:51-135, DistributedClusterSession.cs:1123) -- with
// ncclSend/ncclRecv of the 32-byte header and the wire payload between GPUs.
//
// NCCL is loaded with dlopen at the first call that needs it ("libnccl.so.2":
// in a process that already loaded one, e.g. torch's, that copy is reused),
// so the library has no link-time dependency on it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>
#include <vector>

#include "../../../../include/glacier_b200.h"
#include "kernels.h"

namespace glc {
int set_last_error(int code, const char* msg);
}

namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
    ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*GroupStart)() = nullptr;
    ncclResult_t (*GroupEnd)() = nullptr;
    const char* (*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
    std::string why;
};

const NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!lib) {
            api.why = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        auto sym = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(lib, name));
            return fn != nullptr;
        };
        if (!sym(api.GetUniqueId, "ncclGetUniqueId") || !sym(api.CommInitRank, "ncclCommInitRank") ||
            !sym(api.CommDestroy, "ncclCommDestroy") || !sym(api.Send, "ncclSend") ||
            !sym(api.Recv, "ncclRecv") || !sym(api.GroupStart, "ncclGroupStart") ||
            !sym(api.GroupEnd, "ncclGroupEnd") || !sym(api.GetErrorString, "ncclGetErrorString")) {
            api.why = "libnccl.so.2 lacks a required symbol";
            return;
        }
        api.ok = true;
    });
    return api;
}

int fail(int code, const std::string& msg) { return glc::set_last_error(code, msg.c_str()); }

int nccl_fail(ncclResult_t r, const char* what) {
    return fail(GLC_ERR_NCCL, std::string(what) + ": " + nccl().GetErrorString(r));
}

#define NCCL_TRY(call, what)                               \
    do {                                                   \
        const ncclResult_t r_ = (call);                    \
        if (r_ != ncclSuccess) return nccl_fail(r_, what); \
    } while (0)

#define CUDA_OK(call)                                                                                       \
    do {                                                                                                    \
        const cudaError_t e_ = (call);                                                                      \
        if (e_ != cudaSuccess) return fail(GLC_ERR_CUDA, std::string(#call ": ") + cudaGetErrorString(e_)); \
    } while (0)

}  // namespace

struct glc_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0;
    cudaStream_t stream = nullptr;
    uint8_t* d_hdr = nullptr;  // 64 B: [0, 32) send header, [32, 64) received header
    uint8_t* h_hdr = nullptr;  // pinned copy of a received header
    // device scratch, grown on demand (slot -> buffer)
    std::vector<void*> scratch;
    std::vector<size_t> scratch_bytes;
    std::vector<void*> retired;  // outgrown scratch, possibly still in use by queued work: freed at destroy
    int32_t* h_counts = nullptr;  // pinned [2 * nranks]: counts sent, counts received
    // Peer window (comm_window): this rank's buffer, every rank's buffer
    // mapped into this process (CUDA IPC over NVLink), epochs of the
    // exchanges made through it.  state 0 = not set up, 1 = mapped,
    // -1 = unavailable or turned off (exchanges go through NCCL).
    uint8_t* win = nullptr;
    size_t win_bytes = 0;
    std::vector<void*> win_peer;        // [nranks] host table (own buffer at [rank])
    void** d_win_peer = nullptr;        // device copy of the table
    std::vector<void*> win_mapped;      // peers' mappings to close at destroy
    std::vector<void*> win_retired;     // outgrown own buffers (peers may still hold mappings)
    unsigned long long win_epoch = 0;
    int win_state = 0;
    bool win_enabled = true;
};

namespace glc {

int comm_world(const glc_comm* c) { return c->nranks; }
int comm_rank(const glc_comm* c) { return c->rank; }
int32_t* comm_host_counts(glc_comm* c) { return c->h_counts; }

// Device buffer `slot` of at least `bytes`.  The callers' sizes depend only
// on the handle and the world size, so a slot is allocated by the first call
// and reused; a buffer that must grow is retired, not freed (work already
// queued may still use it), and retired buffers are freed when the
// communicator is destroyed -- no device-wide synchronisation on the way.
void* comm_scratch(glc_comm* c, int slot, size_t bytes) {
    if ((int)c->scratch.size() <= slot) {
        c->scratch.resize(slot + 1, nullptr);
        c->scratch_bytes.resize(slot + 1, 0);
    }
    if (c->scratch_bytes[slot] < bytes) {
        if (c->scratch[slot]) {
            c->retired.push_back(c->scratch[slot]);
            c->scratch[slot] = nullptr;
            c->scratch_bytes[slot] = 0;
        }
        const size_t b = bytes < 256 ? 256 : bytes;
        if (cudaMalloc(&c->scratch[slot], b) != cudaSuccess) return nullptr;
        c->scratch_bytes[slot] = b;
    }
    return c->scratch[slot];
}

// One int32 to and from every rank (send[p] goes to rank p, recv[p] comes from it).
int comm_alltoall_i32(glc_comm* c, const int32_t* send, int32_t* recv, cudaStream_t st) {
    const NcclApi& n = nccl();
    NCCL_TRY(n.GroupStart(), "ncclGroupStart");
    for (int p = 0; p < c->nranks; ++p) {
        NCCL_TRY(n.Send(send + p, 1, ncclInt32, p, c->comm, st), "ncclSend");
        NCCL_TRY(n.Recv(recv + p, 1, ncclInt32, p, c->comm, st), "ncclRecv");
    }
    NCCL_TRY(n.GroupEnd(), "ncclGroupEnd");
    return GLC_OK;
}

// Variable-size blocks to and from every rank: bytes [soff[p], soff[p]+scnt[p])
// of send go to rank p, bytes from rank p land at [roff[p], roff[p]+rcnt[p]).
int comm_alltoallv(glc_comm* c, const void* send, const size_t* soff, const size_t* scnt, void* recv,
                   const size_t* roff, const size_t* rcnt, cudaStream_t st) {
    const NcclApi& n = nccl();
    const uint8_t* s = static_cast<const uint8_t*>(send);
    uint8_t* r = static_cast<uint8_t*>(recv);
    NCCL_TRY(n.GroupStart(), "ncclGroupStart");
    for (int p = 0; p < c->nranks; ++p) {
        if (scnt[p]) NCCL_TRY(n.Send(s + soff[p], scnt[p], ncclUint8, p, c->comm, st), "ncclSend");
        if (rcnt[p]) NCCL_TRY(n.Recv(r + roff[p], rcnt[p], ncclUint8, p, c->comm, st), "ncclRecv");
    }
    NCCL_TRY(n.GroupEnd(), "ncclGroupEnd");
    return GLC_OK;
}

// Peer window of at least `bytes` on every rank (collective: every rank calls
// it with the same size, in the same order as its other exchanges).  The
// buffer is cudaMalloc'd and zeroed, its CUDA IPC handle and size go to every
// peer (a grouped send/receive of 128 bytes each way), each peer's buffer is
// opened in this process (peer access over NVLink), and the ranks agree --
// one int32 each way -- that every rank mapped every peer at the same size;
// if any did not, no rank uses the window (GLC_ERR_UNSUPPORTED: the callers
// exchange through NCCL instead).  A window that must grow is retired, not
// freed: peers may still hold mappings of it and queued work may still use it.
int comm_window(glc_comm* c, size_t bytes, cudaStream_t st, uint8_t** own, void* const** d_peers) {
    if (!c->win_enabled || c->win_state < 0) return GLC_ERR_UNSUPPORTED;
    if (c->win_state == 1 && c->win_bytes >= bytes) {
        *own = c->win;
        *d_peers = c->d_win_peer;
        return GLC_OK;
    }
    const int W = c->nranks, me = c->rank;
    if (c->win) c->win_retired.push_back(c->win);
    c->win = nullptr;
    c->win_state = 0;
    bytes = (bytes + 4095) & ~size_t(4095);
    if (cudaMalloc(&c->win, bytes) != cudaSuccess) return fail(GLC_ERR_OOM, "peer window");
    CUDA_OK(cudaMemset(c->win, 0, bytes));  // flags start at epoch 0 (synchronous: before any peer can write)
    struct Msg {
        cudaIpcMemHandle_t h;
        unsigned long long bytes;
        uint8_t pad[128 - sizeof(cudaIpcMemHandle_t) - 8];
    };
    static_assert(sizeof(Msg) == 128, "window message");
    Msg m{};
    CUDA_OK(cudaIpcGetMemHandle(&m.h, c->win));
    m.bytes = bytes;
    uint8_t* dmsg = static_cast<uint8_t*>(comm_scratch(c, 30, (size_t)(W + 1) * sizeof(Msg) + 64 * (size_t)W * 2));
    if (!dmsg) return fail(GLC_ERR_OOM, "window handles");
    CUDA_OK(cudaMemcpyAsync(dmsg + (size_t)W * sizeof(Msg), &m, sizeof(Msg), cudaMemcpyHostToDevice, st));
    const NcclApi& n = nccl();
    NCCL_TRY(n.GroupStart(), "ncclGroupStart");
    for (int p = 0; p < W; ++p) {
        NCCL_TRY(n.Send(dmsg + (size_t)W * sizeof(Msg), sizeof(Msg), ncclUint8, p, c->comm, st), "ncclSend");
        NCCL_TRY(n.Recv(dmsg + (size_t)p * sizeof(Msg), sizeof(Msg), ncclUint8, p, c->comm, st), "ncclRecv");
    }
    NCCL_TRY(n.GroupEnd(), "ncclGroupEnd");
    std::vector<Msg> all(W);
    CUDA_OK(cudaMemcpyAsync(all.data(), dmsg, (size_t)W * sizeof(Msg), cudaMemcpyDeviceToHost, st));
    CUDA_OK(cudaStreamSynchronize(st));
    std::vector<void*> peer(W, nullptr);
    int ok = 1;
    for (int p = 0; p < W; ++p) {
        if (all[p].bytes != bytes) ok = 0;
        if (p == me) {
            peer[p] = c->win;
            continue;
        }
        if (!ok) continue;
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, all[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
            (void)cudaGetLastError();
            ok = 0;
            continue;
        }
        peer[p] = ptr;
        c->win_mapped.push_back(ptr);
    }
    // every rank's verdict to every rank
    int32_t* dok = reinterpret_cast<int32_t*>(dmsg + (size_t)(W + 1) * sizeof(Msg));
    std::vector<int32_t> mine(W, ok), theirs(W, 0);
    CUDA_OK(cudaMemcpyAsync(dok, mine.data(), sizeof(int32_t) * W, cudaMemcpyHostToDevice, st));
    int rc = comm_alltoall_i32(c, dok, dok + W, st);
    if (rc) return rc;
    CUDA_OK(cudaMemcpyAsync(theirs.data(), dok + W, sizeof(int32_t) * W, cudaMemcpyDeviceToHost, st));
    CUDA_OK(cudaStreamSynchronize(st));
    for (int p = 0; p < W; ++p) ok &= theirs[p] ? 1 : 0;
    if (!ok) {
        c->win_state = -1;
        return GLC_ERR_UNSUPPORTED;
    }
    if (!c->d_win_peer && cudaMalloc(&c->d_win_peer, sizeof(void*) * 64) != cudaSuccess)
        return fail(GLC_ERR_OOM, "peer table");
    CUDA_OK(cudaMemcpy(c->d_win_peer, peer.data(), sizeof(void*) * W, cudaMemcpyHostToDevice));
    c->win_peer = peer;
    c->win_bytes = bytes;
    c->win_state = 1;
    *own = c->win;
    *d_peers = c->d_win_peer;
    return GLC_OK;
}

// Epoch of the next exchange through the peer window (1, 2, ...; every rank
// makes the same exchanges in the same order, so the ranks agree on it).
unsigned long long comm_window_next_epoch(glc_comm* c) { return ++c->win_epoch; }

}  // namespace glc

extern "C" {

int glc_comm_peer_exchange(glc_comm* c, int32_t enable) {
    if (!c) return fail(GLC_ERR_INVALID_ARG, "null communicator");
    if (enable < 0) return (c->win_enabled && c->win_state == 1) ? 1 : 0;
    c->win_enabled = enable != 0;
    return GLC_OK;
}


int glc_comm_unique_id(uint8_t* id_out) {
    if (!id_out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    const NcclApi& n = nccl();
    if (!n.ok) return fail(GLC_ERR_NCCL, n.why);
    static_assert(sizeof(ncclUniqueId) == GLC_COMM_ID_BYTES, "NCCL unique id size");
    ncclUniqueId id;
    NCCL_TRY(n.GetUniqueId(&id), "ncclGetUniqueId");
    std::memcpy(id_out, &id, sizeof(id));
    return GLC_OK;
}

int glc_comm_create(const uint8_t* id, int32_t nranks, int32_t rank, int32_t device, glc_comm** out) {
    if (!id || !out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    *out = nullptr;
    if (nranks < 1 || rank < 0 || rank >= nranks) return fail(GLC_ERR_INVALID_ARG, "rank out of range");
    const NcclApi& n = nccl();
    if (!n.ok) return fail(GLC_ERR_NCCL, n.why);
    CUDA_OK(cudaSetDevice(device));
    glc_comm* c = new glc_comm();
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    auto cleanup = [&](int rc) { glc_comm_destroy(c); return rc; };
    if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&c->d_hdr, 64) != cudaSuccess || cudaMallocHost(&c->h_hdr, 64) != cudaSuccess ||
        cudaMallocHost(&c->h_counts, sizeof(int32_t) * 2 * nranks) != cudaSuccess)
        return cleanup(fail(GLC_ERR_OOM, "communicator buffers"));
    ncclUniqueId uid;
    std::memcpy(&uid, id, sizeof(uid));
    const ncclResult_t r = n.CommInitRank(&c->comm, nranks, uid, rank);
    if (r != ncclSuccess) {
        c->comm = nullptr;
        return cleanup(nccl_fail(r, "ncclCommInitRank"));
    }
    *out = c;
    return GLC_OK;
}

int glc_comm_destroy(glc_comm* c) {
    if (!c) return GLC_OK;
    cudaSetDevice(c->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->comm) nccl().CommDestroy(c->comm);
    cudaDeviceSynchronize();  // work of other streams may still use the scratch
    for (void* p : c->win_mapped) cudaIpcCloseMemHandle(p);
    for (void* p : c->win_retired) cudaFree(p);
    cudaFree(c->win);
    cudaFree(c->d_win_peer);
    for (void* p : c->scratch) cudaFree(p);
    for (void* p : c->retired) cudaFree(p);
    cudaFree(c->d_hdr);
    cudaFreeHost(c->h_hdr);
    cudaFreeHost(c->h_counts);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    return GLC_OK;
}

int glc_pp_send(glc_comm* c, int32_t peer, const glc_fused_header* hdr, const float* x, void* stream) {
    if (!c || !hdr || !x) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (peer < 0 || peer >= c->nranks || peer == c->rank) return fail(GLC_ERR_INVALID_ARG, "bad peer rank");
    if (hdr->flags & 0x10) return fail(GLC_ERR_UNSUPPORTED, "token-id payloads (Stage0TokenInput) are not sent here");
    const int mode = hdr->precision_mode, D = hdr->hidden_dim;
    const int T = hdr->batch_tokens > 0 ? hdr->batch_tokens : 1;
    const int32_t tb = glc_wire_token_bytes(mode, D);
    if (tb <= 0 || D <= 0) return fail(GLC_ERR_INVALID_ARG, "bad precision mode or hidden dim");
    const size_t payload = (size_t)T * tb;
    CUDA_OK(cudaSetDevice(c->device));
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    uint8_t hb[32];
    int rc = glc_fused_header_write(hdr, hb);
    if (rc) return rc;
    // from a pageable buffer: returns once the bytes are staged, so hb may go
    CUDA_OK(cudaMemcpyAsync(c->d_hdr, hb, 32, cudaMemcpyHostToDevice, st));
    uint8_t* dp = static_cast<uint8_t*>(glc::comm_scratch(c, 0, payload));
    if (!dp) return fail(GLC_ERR_OOM, "payload staging");
    CUDA_OK(glc::wire_quantize_launch(mode, x, T, D, dp, st));
    const NcclApi& n = nccl();
    NCCL_TRY(n.Send(c->d_hdr, 32, ncclUint8, peer, c->comm, st), "ncclSend (header)");
    NCCL_TRY(n.Send(dp, payload, ncclUint8, peer, c->comm, st), "ncclSend (payload)");
    return GLC_OK;
}

int glc_pp_recv(glc_comm* c, int32_t peer, glc_fused_header* hdr_out, float* x_out, int32_t max_tokens,
                int32_t hidden_dim, void* stream) {
    if (!c || !hdr_out || !x_out) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (peer < 0 || peer >= c->nranks || peer == c->rank) return fail(GLC_ERR_INVALID_ARG, "bad peer rank");
    CUDA_OK(cudaSetDevice(c->device));
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    const NcclApi& n = nccl();
    NCCL_TRY(n.Recv(c->d_hdr + 32, 32, ncclUint8, peer, c->comm, st), "ncclRecv (header)");
    CUDA_OK(cudaMemcpyAsync(c->h_hdr, c->d_hdr + 32, 32, cudaMemcpyDeviceToHost, st));
    CUDA_OK(cudaStreamSynchronize(st));
    int rc = glc_fused_header_read(c->h_hdr, hdr_out);
    if (rc) return rc;  // not a header: the sender's payload cannot be sized, as in the reference
    const int32_t pb = glc_fused_header_payload_bytes(hdr_out);
    const int T = hdr_out->batch_tokens > 0 ? hdr_out->batch_tokens : 1;
    uint8_t* dp = static_cast<uint8_t*>(glc::comm_scratch(c, 1, pb > 0 ? (size_t)pb : 16));
    if (!dp) return fail(GLC_ERR_OOM, "payload staging");
    // the payload is taken off the link even when it cannot be used, so the
    // next message on this link still lines up
    if (pb > 0) NCCL_TRY(n.Recv(dp, (size_t)pb, ncclUint8, peer, c->comm, st), "ncclRecv (payload)");
    if (hdr_out->flags & 0x10) return fail(GLC_ERR_UNSUPPORTED, "token-id payloads (Stage0TokenInput) are not decoded here");
    if (hdr_out->hidden_dim != hidden_dim || T > max_tokens)
        return fail(GLC_ERR_INVALID_ARG, "message of " + std::to_string(T) + " x " + std::to_string(hdr_out->hidden_dim) +
                                             " does not fit the receive buffer");
    CUDA_OK(glc::wire_dequantize_launch(hdr_out->precision_mode, dp, T, hidden_dim, x_out, st));
    return GLC_OK;
}

int glc_comm_send(glc_comm* c, int32_t peer, const void* buf, size_t bytes, void* stream) {
    if (!c || (!buf && bytes)) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (peer < 0 || peer >= c->nranks || peer == c->rank) return fail(GLC_ERR_INVALID_ARG, "bad peer rank");
    if (!bytes) return GLC_OK;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    NCCL_TRY(nccl().Send(buf, bytes, ncclUint8, peer, c->comm, st), "ncclSend");
    return GLC_OK;
}

int glc_comm_recv(glc_comm* c, int32_t peer, void* buf, size_t bytes, void* stream) {
    if (!c || (!buf && bytes)) return fail(GLC_ERR_INVALID_ARG, "null pointer");
    if (peer < 0 || peer >= c->nranks || peer == c->rank) return fail(GLC_ERR_INVALID_ARG, "bad peer rank");
    if (!bytes) return GLC_OK;
    cudaStream_t st = stream ? (cudaStream_t)stream : c->stream;
    NCCL_TRY(nccl().Recv(buf, bytes, ncclUint8, peer, c->comm, st), "ncclRecv");
    return GLC_OK;
}

}  // extern "C"
