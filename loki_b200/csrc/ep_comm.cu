// ep_comm.cu -- the expert-parallel exchange: an NCCL communicator over the node's GPUs and the
// all-to-all of row blocks (grouped ncclSend / ncclRecv, one pair per peer; the block a rank keeps is a
// device copy).  Stream-ordered and CUDA-graph capturable (NCCL point-to-point calls are captured as
// graph nodes), so a decode step's exchanges sit inside the step's graph.
//
// libnccl.so.2 is bound at run time (the copy a host process already loaded, e.g. PyTorch's, else the
// system one): the library has no link-time NCCL dependency, and one NCCL serves the whole process.
#include <dlfcn.h>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <nccl.h>
#include "../../include/loki_ep.h"

namespace {

struct NcclApi {
    ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*group_start)() = nullptr;
    ncclResult_t (*group_end)() = nullptr;
    const char* (*error_string)(ncclResult_t) = nullptr;
    bool ok = false;
};

NcclApi& nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) { fprintf(stderr, "loki_ep: libnccl.so.2 not found: %s\n", dlerror()); return; }
        api.get_unique_id = (decltype(api.get_unique_id))dlsym(h, "ncclGetUniqueId");
        api.comm_init_rank = (decltype(api.comm_init_rank))dlsym(h, "ncclCommInitRank");
        api.comm_destroy = (decltype(api.comm_destroy))dlsym(h, "ncclCommDestroy");
        api.send = (decltype(api.send))dlsym(h, "ncclSend");
        api.recv = (decltype(api.recv))dlsym(h, "ncclRecv");
        api.group_start = (decltype(api.group_start))dlsym(h, "ncclGroupStart");
        api.group_end = (decltype(api.group_end))dlsym(h, "ncclGroupEnd");
        api.error_string = (decltype(api.error_string))dlsym(h, "ncclGetErrorString");
        api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.send && api.recv && api.group_start &&
                 api.group_end && api.error_string;
        if (!api.ok) fprintf(stderr, "loki_ep: libnccl.so.2 lacks point-to-point entry points\n");
    });
    return api;
}

int nccl_rc(ncclResult_t r, const char* what) {
    if (r == ncclSuccess) return LK_OK;
    fprintf(stderr, "loki_ep: %s: %s\n", what, nccl().error_string ? nccl().error_string(r) : "nccl error");
    return LK_ERR_CUDA;
}

}  // namespace

struct LkEpComm {
    ncclComm_t comm = nullptr;
    int n_ranks = 0, rank = 0, device = 0;
};

extern "C" {

int lk_ep_comm_id(void* id_out) {
    if (!id_out) return LK_ERR_ARG;
    if (!nccl().ok) return LK_ERR_UNSUPPORTED;
    ncclUniqueId id;
    int rc = nccl_rc(nccl().get_unique_id(&id), "ncclGetUniqueId");
    if (rc) return rc;
    memcpy(id_out, &id, sizeof(id));
    return LK_OK;
}

int lk_ep_comm_create(const void* id, int n_ranks, int rank, int device, LkEpComm** out) {
    if (!id || !out || n_ranks < 1 || n_ranks > LK_EP_MAX_RANKS || rank < 0 || rank >= n_ranks) return LK_ERR_ARG;
    *out = nullptr;
    if (!nccl().ok) return LK_ERR_UNSUPPORTED;
    if (cudaSetDevice(device) != cudaSuccess) return LK_ERR_CUDA;
    ncclUniqueId uid;
    memcpy(&uid, id, sizeof(uid));
    LkEpComm* c = new LkEpComm();
    c->n_ranks = n_ranks; c->rank = rank; c->device = device;
    int rc = nccl_rc(nccl().comm_init_rank(&c->comm, n_ranks, uid, rank), "ncclCommInitRank");
    if (rc) { delete c; return rc; }
    *out = c;
    return LK_OK;
}

void lk_ep_comm_destroy(LkEpComm* c) {
    if (!c) return;
    if (c->comm) nccl().comm_destroy(c->comm);
    delete c;
}

int lk_ep_all_to_all(LkEpComm* c, const void* send, void* recv, const int64_t* send_off, const int64_t* send_bytes,
                     const int64_t* recv_off, const int64_t* recv_bytes, int64_t block_bytes, lk_stream_t stream) {
    if (!c || (!send_bytes != !recv_bytes) || (!send_off != !send_bytes) || (!recv_off != !recv_bytes)) return LK_ERR_ARG;
    if (!send_bytes && block_bytes < 0) return LK_ERR_ARG;
    cudaStream_t st = (cudaStream_t)stream;
    const int n = c->n_ranks, me = c->rank;
    auto soff = [&](int d) { return send_off ? send_off[d] : (int64_t)d * block_bytes; };
    auto sbytes = [&](int d) { return send_bytes ? send_bytes[d] : block_bytes; };
    auto roff = [&](int s) { return recv_off ? recv_off[s] : (int64_t)s * block_bytes; };
    auto rbytes = [&](int s) { return recv_bytes ? recv_bytes[s] : block_bytes; };
    for (int d = 0; d < n; ++d)
        if (sbytes(d) < 0 || rbytes(d) < 0 || ((sbytes(d) || rbytes(d)) && (!send || !recv))) return LK_ERR_ARG;
    if (sbytes(me) != rbytes(me)) return LK_ERR_ARG;
    if (sbytes(me) > 0 && cudaMemcpyAsync((uint8_t*)recv + roff(me), (const uint8_t*)send + soff(me), (size_t)sbytes(me),
                                          cudaMemcpyDeviceToDevice, st) != cudaSuccess)
        return LK_ERR_CUDA;
    if (n == 1) return LK_OK;
    int rc = nccl_rc(nccl().group_start(), "ncclGroupStart");
    if (rc) return rc;
    for (int k = 1; k < n; ++k) {                  // peers in a rotating order: rank me+k receives while me-k sends
        const int to = (me + k) % n, from = (me - k + n) % n;
        if (sbytes(to) > 0)
            rc |= nccl_rc(nccl().send((const uint8_t*)send + soff(to), (size_t)sbytes(to), ncclUint8, to, c->comm, st), "ncclSend");
        if (rbytes(from) > 0)
            rc |= nccl_rc(nccl().recv((uint8_t*)recv + roff(from), (size_t)rbytes(from), ncclUint8, from, c->comm, st), "ncclRecv");
    }
    int rc2 = nccl_rc(nccl().group_end(), "ncclGroupEnd");
    return rc ? LK_ERR_CUDA : rc2;
}

}  // extern "C"
