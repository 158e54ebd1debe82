// Expert parallelism inside the library: one NCCL communicator per context.
//
// A context that joined a communicator (moe_ep_init) evaluates, in
// moe_layer_forward, only the experts of its rank's contiguous range
// [rank*E/N, (rank+1)*E/N), all-reduces the partial outputs of all ranks in
// place on its stream, and applies the post-norm to the sum: every rank
// passes the same tokens and gets the whole layer's output (the decode form,
// where an all-reduce of M x d fp32 costs less than exchanging the routed
// rows).  This is what a host that is not Python (the reference's Mojo
// engine) needs to run the layer on several GPUs through the C ABI alone.
//
// NCCL is resolved with dlopen at the first moe_ep_* call, so the library
// loads on hosts without it.  The communicator is non-blocking: its
// creation and every collective are polled with a deadline, and a
// communicator that reports an error or misses the deadline is aborted, so
// no host wait in this file is unbounded and a rank that left makes the
// others fail with a status instead of hanging.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstring>
#include <mutex>
#include <string>
#include <thread>
#include <type_traits>
#include <vector>

#include "moe_b200.h"
#include "moe_internal.h"

namespace {

struct NcclApi {
    decltype(&ncclGetUniqueId) get_unique_id = nullptr;
    decltype(&ncclCommInitRankConfig) init_rank_config = nullptr;
    decltype(&ncclAllReduce) all_reduce = nullptr;
    decltype(&ncclAllGather) all_gather = nullptr;
    decltype(&ncclReduceScatter) reduce_scatter = nullptr;
    decltype(&ncclSend) send = nullptr;
    decltype(&ncclRecv) recv = nullptr;
    decltype(&ncclGroupStart) group_start = nullptr;
    decltype(&ncclGroupEnd) group_end = nullptr;
    decltype(&ncclCommDestroy) destroy = nullptr;
    decltype(&ncclCommAbort) abort = nullptr;
    decltype(&ncclCommGetAsyncError) async_error = nullptr;
    decltype(&ncclGetErrorString) error_string = nullptr;
};

const NcclApi* nccl(std::string& err) {
    static NcclApi api;
    static bool ok = false;
    static std::string load_err;
    static std::once_flag once;
    std::call_once(once, [] {
        // an NCCL already in the process (e.g. loaded by the host's own
        // framework) is found first under its soname
        void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) h = dlopen("libnccl.so", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            load_err = std::string("cannot load libnccl.so.2: ") + dlerror();
            return;
        }
        auto get = [&](auto& fn, const char* name) {
            fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name));
            if (!fn && load_err.empty()) load_err = std::string("libnccl lacks ") + name;
        };
        get(api.get_unique_id, "ncclGetUniqueId");
        get(api.init_rank_config, "ncclCommInitRankConfig");
        get(api.all_reduce, "ncclAllReduce");
        get(api.all_gather, "ncclAllGather");
        get(api.reduce_scatter, "ncclReduceScatter");
        get(api.send, "ncclSend");
        get(api.recv, "ncclRecv");
        get(api.group_start, "ncclGroupStart");
        get(api.group_end, "ncclGroupEnd");
        get(api.destroy, "ncclCommDestroy");
        get(api.abort, "ncclCommAbort");
        get(api.async_error, "ncclCommGetAsyncError");
        get(api.error_string, "ncclGetErrorString");
        ok = load_err.empty();
    });
    if (!ok) {
        err = load_err;
        return nullptr;
    }
    return &api;
}

uint64_t now_ns() {
    return (uint64_t)std::chrono::duration_cast<std::chrono::nanoseconds>(
               std::chrono::steady_clock::now().time_since_epoch())
        .count();
}

std::string nccl_msg(const NcclApi* api, const char* what, ncclResult_t r) {
    return std::string(what) + ": " + (api->error_string ? api->error_string(r) : "NCCL error");
}

// Polls the communicator until its pending operation left ncclInProgress.
// An enqueue usually settles within microseconds: the first 200 us poll
// without sleeping, so that a layer call does not stall its host thread
// (and, with eager launches, the GPU behind it) for a whole sleep.
int settle(moe::EpComm& ep, const NcclApi* api, uint64_t deadline, const char* what, std::string& err) {
    ncclComm_t comm = static_cast<ncclComm_t>(ep.comm);
    const uint64_t spin_until = now_ns() + 200000;
    for (;;) {
        ncclResult_t st = ncclInProgress;
        ncclResult_t r = api->async_error(comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return MOE_OK;
        if (st != ncclInProgress) {
            err = nccl_msg(api, what, st);
            moe::ep_abort(ep);
            return MOE_E_NCCL;
        }
        const uint64_t t = now_ns();
        if (t > deadline) {
            err = std::string(what) + ": no progress before the deadline (a rank missing?)";
            moe::ep_abort(ep);
            return MOE_E_TIMEOUT;
        }
        if (t < spin_until)
            std::this_thread::yield();
        else
            std::this_thread::sleep_for(std::chrono::microseconds(50));
    }
}

}  // namespace

namespace moe {

int ep_unique_id(uint8_t* out, std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api) return MOE_E_NCCL;
    ncclUniqueId id;
    ncclResult_t r = api->get_unique_id(&id);
    if (r != ncclSuccess) {
        err = nccl_msg(api, "ncclGetUniqueId", r);
        return MOE_E_NCCL;
    }
    static_assert(sizeof(id.internal) == MOE_EP_UNIQUE_ID_BYTES, "NCCL unique id size");
    std::memcpy(out, id.internal, sizeof(id.internal));
    return MOE_OK;
}

int ep_init(EpComm& ep, const uint8_t* id, int rank, int nranks, uint64_t timeout_ns, std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api) return MOE_E_NCCL;
    ncclUniqueId uid;
    std::memcpy(uid.internal, id, sizeof(uid.internal));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // returns at once; progress is polled below
    ncclComm_t comm = nullptr;
    ncclResult_t r = api->init_rank_config(&comm, nranks, uid, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        err = nccl_msg(api, "ncclCommInitRankConfig", r);
        if (comm) api->abort(comm);
        return MOE_E_NCCL;
    }
    ep.comm = comm;
    ep.rank = rank;
    ep.nranks = nranks;
    ep.pending = false;
    return settle(ep, api, now_ns() + timeout_ns, "NCCL communicator set-up", err);
}

int ep_all_reduce(EpComm& ep, float* buf, size_t count, cudaStream_t s, uint64_t timeout_ns, std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api || !ep.comm) {
        if (api) err = "no expert-parallel communicator";
        return MOE_E_STATE;
    }
    ncclResult_t r = api->all_reduce(buf, buf, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(ep.comm), s);
    if (r != ncclSuccess && r != ncclInProgress) {
        err = nccl_msg(api, "ncclAllReduce", r);
        ep_abort(ep);
        return MOE_E_NCCL;
    }
    if (r == ncclInProgress) {
        const int s2 = settle(ep, api, now_ns() + timeout_ns, "ncclAllReduce", err);
        if (s2 != MOE_OK) return s2;
    }
    ep.pending = true;
    return MOE_OK;
}

namespace {
// Common tail of an enqueue: an error aborts the communicator, an enqueue
// still in progress is polled to completion, and the context is marked as
// having a collective in flight.
int enqueued(EpComm& ep, const NcclApi* api, ncclResult_t r, const char* what, uint64_t timeout_ns, std::string& err) {
    if (r != ncclSuccess && r != ncclInProgress) {
        err = nccl_msg(api, what, r);
        ep_abort(ep);
        return MOE_E_NCCL;
    }
    if (r == ncclInProgress) {
        const int s2 = settle(ep, api, now_ns() + timeout_ns, what, err);
        if (s2 != MOE_OK) return s2;
    }
    ep.pending = true;
    return MOE_OK;
}
}  // namespace

int ep_all_gather(EpComm& ep, const void* send, void* recv, size_t count, bool is_float, cudaStream_t s,
                  uint64_t timeout_ns, std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api || !ep.comm) {
        if (api) err = "no expert-parallel communicator";
        return MOE_E_STATE;
    }
    const ncclResult_t r = api->all_gather(send, recv, count, is_float ? ncclFloat32 : ncclInt32,
                                           static_cast<ncclComm_t>(ep.comm), s);
    return enqueued(ep, api, r, "ncclAllGather", timeout_ns, err);
}

int ep_all_gather_n(EpComm& ep, const EpGatherBuf* bufs, int n, cudaStream_t s, uint64_t timeout_ns,
                    std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api || !ep.comm) {
        if (api) err = "no expert-parallel communicator";
        return MOE_E_STATE;
    }
    ncclComm_t comm = static_cast<ncclComm_t>(ep.comm);
    ncclResult_t r = api->group_start();
    if (r != ncclSuccess) return enqueued(ep, api, r, "ncclGroupStart", timeout_ns, err);
    for (int i = 0; i < n; ++i) {
        r = api->all_gather(bufs[i].send, bufs[i].recv, bufs[i].count, bufs[i].is_float ? ncclFloat32 : ncclInt32,
                            comm, s);
        if (r != ncclSuccess && r != ncclInProgress) break;
    }
    const ncclResult_t r2 = api->group_end();
    if (r != ncclSuccess && r != ncclInProgress) {
        err = nccl_msg(api, "ncclAllGather", r);
        ep_abort(ep);
        return MOE_E_NCCL;
    }
    return enqueued(ep, api, r2, "ncclGroupEnd (all-gather)", timeout_ns, err);
}

int ep_reduce_scatter(EpComm& ep, const float* send, float* recv, size_t count, cudaStream_t s, uint64_t timeout_ns,
                      std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api || !ep.comm) {
        if (api) err = "no expert-parallel communicator";
        return MOE_E_STATE;
    }
    const ncclResult_t r =
        api->reduce_scatter(send, recv, count, ncclFloat32, ncclSum, static_cast<ncclComm_t>(ep.comm), s);
    return enqueued(ep, api, r, "ncclReduceScatter", timeout_ns, err);
}

int ep_exchange(EpComm& ep, const std::vector<EpXfer>& xfers, cudaStream_t s, uint64_t timeout_ns, std::string& err) {
    const NcclApi* api = nccl(err);
    if (!api || !ep.comm) {
        if (api) err = "no expert-parallel communicator";
        return MOE_E_STATE;
    }
    ncclComm_t comm = static_cast<ncclComm_t>(ep.comm);
    ncclResult_t r = api->group_start();
    if (r != ncclSuccess) return enqueued(ep, api, r, "ncclGroupStart", timeout_ns, err);
    for (const EpXfer& x : xfers) {
        if (x.count == 0) continue;
        const ncclDataType_t dt = x.is_float ? ncclFloat32 : ncclInt32;
        r = x.send ? api->send(x.buf, x.count, dt, x.peer, comm, s) : api->recv(x.buf, x.count, dt, x.peer, comm, s);
        if (r != ncclSuccess && r != ncclInProgress) break;
    }
    const ncclResult_t r2 = api->group_end();
    if (r != ncclSuccess && r != ncclInProgress) {
        err = nccl_msg(api, "ncclSend/ncclRecv", r);
        ep_abort(ep);
        return MOE_E_NCCL;
    }
    return enqueued(ep, api, r2, "ncclGroupEnd (send/recv)", timeout_ns, err);
}

int ep_wait(EpComm& ep, cudaEvent_t done, uint64_t timeout_ns, bool abort_on_timeout, std::string& err) {
    std::string e2;
    const NcclApi* api = nccl(e2);
    const uint64_t deadline = now_ns() + timeout_ns;
    for (;;) {
        cudaError_t e = cudaEventQuery(done);
        if (e == cudaSuccess) {
            ep.pending = false;
            return MOE_OK;
        }
        if (e != cudaErrorNotReady) {
            err = std::string("waiting for a collective: ") + cudaGetErrorString(e);
            return MOE_E_CUDA;
        }
        if (api && ep.comm) {
            ncclResult_t st = ncclSuccess;
            if (api->async_error(static_cast<ncclComm_t>(ep.comm), &st) == ncclSuccess && st != ncclSuccess &&
                st != ncclInProgress) {
                err = nccl_msg(api, "expert-parallel collective", st);
                ep_abort(ep);
                return MOE_E_NCCL;
            }
        }
        if (now_ns() > deadline) {
            err = "expert-parallel collective did not complete before the deadline (a rank missing?)";
            if (abort_on_timeout) ep_abort(ep);
            return MOE_E_TIMEOUT;
        }
        std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
}

void ep_abort(EpComm& ep) {
    std::string err;
    const NcclApi* api = nccl(err);
    if (api && ep.comm) api->abort(static_cast<ncclComm_t>(ep.comm));
    ep.comm = nullptr;
    ep.nranks = 0;
    ep.pending = false;
}

void ep_destroy(EpComm& ep) {
    std::string err;
    const NcclApi* api = nccl(err);
    if (api && ep.comm) api->destroy(static_cast<ncclComm_t>(ep.comm));
    ep.comm = nullptr;
    ep.nranks = 0;
    ep.pending = false;
}

}  // namespace moe
