// seqpar.cu -- the sequence-sharded selective scan as one library call over
// an NCCL communicator: rank r of `world` holds time slice r of every
// sequence.  The recurrence h_t = a_t h_{t-1} + b_t is an affine map per
// (batch, channel, state); a slice applies the composed map h -> P h + H to
// its entering state (the carry monoid of
// Sources/CPURef/selective_scan_cpu.hpp:12-19, at GPU granularity as
// Sources/Kernels/prefix_scan.metal:19-40 intended for tiles).  On the
// caller's stream:
//   1. summary of the local slice: (P, H) [batch, dim, dstate] FP32 (when the
//      slice is split into time chunks, their summaries are kept)
//   2. ncclAllGather of the 2 * batch * dim * dstate floats (the only exchange)
//   3. compose the summaries of ranks < r over the sequence's initial state
//   4. the output pass over the local slice from that state (the kept chunk
//      summaries combined from it), writing y and the slice's final state
// so each slice is read twice, as in a one-GPU chunked scan.
// NCCL is loaded at run time (libnccl.so.2, the copy the process already
// has, e.g. PyTorch's), so the rest of the library works without it.
#include <dlfcn.h>
#include <nccl.h>

#include <cstring>
#include <mutex>
#include <string>

#include "common.cuh"
#include "internal.h"

namespace mb {

namespace {

struct NcclApi {
    bool loaded = false;
    std::string why;
    ncclResult_t (*get_unique_id)(ncclUniqueId *) = nullptr;
    ncclResult_t (*comm_init_rank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int *) = nullptr;
    ncclResult_t (*comm_user_rank)(const ncclComm_t, int *) = nullptr;
    const char *(*error_string)(ncclResult_t) = nullptr;
};

const NcclApi &nccl() {
    static NcclApi api;
    static std::once_flag once;
    std::call_once(once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            api.why = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        auto sym = [&](const char *n) { return dlsym(h, n); };
        api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(sym("ncclGetUniqueId"));
        api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(sym("ncclCommInitRank"));
        api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(sym("ncclCommDestroy"));
        api.all_gather = reinterpret_cast<decltype(api.all_gather)>(sym("ncclAllGather"));
        api.comm_count = reinterpret_cast<decltype(api.comm_count)>(sym("ncclCommCount"));
        api.comm_user_rank = reinterpret_cast<decltype(api.comm_user_rank)>(sym("ncclCommUserRank"));
        api.error_string = reinterpret_cast<decltype(api.error_string)>(sym("ncclGetErrorString"));
        api.loaded = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather &&
                     api.comm_count && api.comm_user_rank && api.error_string;
        if (!api.loaded) api.why = "libnccl.so.2 lacks an expected symbol";
    });
    return api;
}

#define MB_NCCL_TRY(expr, what)                                                                            \
    do {                                                                                                   \
        const ncclResult_t _r = (expr);                                                                    \
        if (_r != ncclSuccess) {                                                                           \
            ::mb::set_error(std::string(what) + ": " + nccl().error_string(_r));                          \
            return -1;                                                                                     \
        }                                                                                                  \
    } while (0)

int need_nccl(const char *what) {
    MB_CHECK_ARG(nccl().loaded, std::string(what) + ": " + nccl().why);
    return 0;
}

size_t align256(size_t v) { return (v + 255) / 256 * 256; }

}  // namespace

size_t seqpar_workspace_bytes(const MambaScanArgs *a, int world) {
    if (!a || world < 1 || a->batch <= 0 || a->dim <= 0) return 0;
    const size_t count = (size_t)a->batch * a->dim * a->dstate;
    return align256(2 * count * 4) + align256((size_t)world * 2 * count * 4) + align256(count * 4) +
           align256(chunked_workspace_bytes(a));
}

int seqpar_scan(const MambaScanArgs *a, void *comm, int world, int rank, void *ws, size_t ws_bytes,
                cudaStream_t st) {
    MB_CHECK_ARG(a != nullptr && comm != nullptr, "selective_scan_seqpar: null args or communicator");
    MB_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "selective_scan_seqpar: bad world or rank");
    if (need_nccl("selective_scan_seqpar")) return -1;
    ncclComm_t c = static_cast<ncclComm_t>(comm);
    int cw = 0, cr = 0;
    MB_NCCL_TRY(nccl().comm_count(c, &cw), "ncclCommCount");
    MB_NCCL_TRY(nccl().comm_user_rank(c, &cr), "ncclCommUserRank");
    MB_CHECK_ARG(cw == world && cr == rank, "selective_scan_seqpar: world/rank differ from the communicator's");
    if (a->batch == 0 || a->dim == 0) return 0;
    const size_t need = seqpar_workspace_bytes(a, world);
    MB_CHECK_ARG(ws != nullptr && ws_bytes >= need,
                 "selective_scan_seqpar: workspace too small (see mamba_selective_scan_seqpar_workspace)");
    MB_CHECK_ARG(reinterpret_cast<uintptr_t>(ws) % 256 == 0, "selective_scan_seqpar: workspace must be 256-byte aligned");
    const size_t count = (size_t)a->batch * a->dim * a->dstate;
    char *p = static_cast<char *>(ws);
    float *local = reinterpret_cast<float *>(p);  // [2][count]: P then H of this slice
    p += align256(2 * count * 4);
    float *all = reinterpret_cast<float *>(p);  // [world][2][count]
    p += align256((size_t)world * 2 * count * 4);
    float *h_in = reinterpret_cast<float *>(p);  // [count]
    p += align256(count * 4);
    void *scan_ws = p;
    const size_t scan_ws_bytes = ws_bytes - (size_t)(p - static_cast<char *>(ws));
    // 1. the slice's summary (independent of its entering state); its chunk
    //    summaries stay in scan_ws for step 4
    if (scan_seqpar_pass1(a, local, local + count, scan_ws, scan_ws_bytes, st)) return -1;
    // 2. every rank's summary
    MB_NCCL_TRY(nccl().all_gather(local, all, 2 * count, ncclFloat32, c, st), "ncclAllGather");
    // 3. the state entering this slice
    if (scan_compose_prefix(all, world, rank, (int64_t)count, a->initial_state, h_in, st)) return -1;
    // 4. the output pass from it (chunk summaries combined, not recomputed)
    MambaScanArgs local_args = *a;
    local_args.initial_state = h_in;
    return scan_seqpar_pass2(&local_args, scan_ws, scan_ws_bytes, st);
}

int nccl_unique_id(void *id) {
    MB_CHECK_ARG(id != nullptr, "nccl_unique_id: null buffer");
    if (need_nccl("nccl_unique_id")) return -1;
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    ncclUniqueId u;
    MB_NCCL_TRY(nccl().get_unique_id(&u), "ncclGetUniqueId");
    std::memcpy(id, &u, sizeof(u));
    return 0;
}

int nccl_comm_create(const void *id, int world, int rank, void **comm) {
    MB_CHECK_ARG(id && comm, "nccl_comm_create: null pointer");
    MB_CHECK_ARG(world >= 1 && rank >= 0 && rank < world, "nccl_comm_create: bad world or rank");
    if (need_nccl("nccl_comm_create")) return -1;
    ncclUniqueId u;
    std::memcpy(&u, id, sizeof(u));
    ncclComm_t c = nullptr;
    MB_NCCL_TRY(nccl().comm_init_rank(&c, world, u, rank), "ncclCommInitRank");
    *comm = c;
    return 0;
}

int nccl_comm_destroy(void *comm) {
    if (!comm) return 0;
    if (need_nccl("nccl_comm_destroy")) return -1;
    MB_NCCL_TRY(nccl().comm_destroy(static_cast<ncclComm_t>(comm)), "ncclCommDestroy");
    return 0;
}

}  // namespace mb
