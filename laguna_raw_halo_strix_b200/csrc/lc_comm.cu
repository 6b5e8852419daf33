// lc_comm.cu -- the vocab-sharded lm_head's reduction over NCCL, owned by the
// library: a communicator per context, the int64 MAX all-reduce of the packed
// (logit, index) keys, and bounded host-side waits.
//
// Reference: TargetModel::project_normalized_hidden (src/target.rs:580-605)
// projects one hidden row onto the whole vocabulary and argmax (src/lib.rs:
// 456-464) takes the last maximum.  Sharded over G GPUs, rank r holds vocab rows
// [lo_r, hi_r); its keys are the shard's best (logit, global index) per token,
// packed so that a signed int64 maximum is the reference's argmax (lc_pack_key),
// and one all-reduce of m keys gives every rank the global draft tokens.
//
// NCCL is opened at run time (dlopen of libnccl.so.2: whatever copy the
// process already holds, else the system's), so the library loads without it
// and only these entry points need it.  The communicator is created
// non-blocking; every wait on it -- its creation and each reduction -- polls
// ncclCommGetAsyncError and the stream against a host deadline, and on expiry
// aborts the communicator (which ends its kernels) and returns LC_ERR_TIMEOUT:
// a rank that never arrives costs the others the timeout, not a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <thread>

#include "lc_internal.cuh"

namespace {

struct NcclApi {
    ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
    ncclResult_t (*CommInitRankConfig)(ncclComm_t *, int, ncclUniqueId, int, ncclConfig_t *) = nullptr;
    ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
    ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                              cudaStream_t) = nullptr;
    ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
    ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
    ncclResult_t (*CommFinalize)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(ncclResult_t) = nullptr;
    bool ok = false;
    char why[256] = "";
};

NcclApi g_nccl;
std::once_flag g_nccl_once;

const NcclApi &nccl() {
    std::call_once(g_nccl_once, [] {
        void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
        if (!h) {
            snprintf(g_nccl.why, sizeof(g_nccl.why), "libnccl.so.2 not found: %s", dlerror());
            return;
        }
#define LC_SYM(f, name)                                                           \
    *reinterpret_cast<void **>(&g_nccl.f) = dlsym(h, name);                      \
    if (!g_nccl.f) {                                                              \
        snprintf(g_nccl.why, sizeof(g_nccl.why), "libnccl.so.2 has no %s", name); \
        return;                                                                   \
    }
        LC_SYM(GetUniqueId, "ncclGetUniqueId")
        LC_SYM(CommInitRankConfig, "ncclCommInitRankConfig")
        LC_SYM(CommGetAsyncError, "ncclCommGetAsyncError")
        LC_SYM(AllReduce, "ncclAllReduce")
        LC_SYM(CommAbort, "ncclCommAbort")
        LC_SYM(CommDestroy, "ncclCommDestroy")
        LC_SYM(CommFinalize, "ncclCommFinalize")
        LC_SYM(GetErrorString, "ncclGetErrorString")
#undef LC_SYM
        g_nccl.ok = true;
    });
    return g_nccl;
}

using Clock = std::chrono::steady_clock;

}  // namespace

struct lc_comm {
    ncclComm_t comm = nullptr;
    int n_ranks = 0, rank = 0, device = 0;
    int timeout_ms = 0;
    bool aborted = false;
};

namespace {

int need_nccl(const char *what) {
    const NcclApi &n = nccl();
    LC_REQUIRE(n.ok, LC_ERR_UNSUPPORTED, "%s: %s", what, n.why);
    return LC_OK;
}

// Abort after a failure or an expired wait; the communicator is unusable after.
void abort_comm(lc_comm *c) {
    if (c->comm && !c->aborted) {
        nccl().CommAbort(c->comm);
        c->aborted = true;
        c->comm = nullptr;
    }
}

// Poll the communicator's asynchronous state until it leaves ncclInProgress,
// within the deadline.
int wait_ready(lc_comm *c, Clock::time_point deadline, const char *what) {
    const NcclApi &n = nccl();
    for (;;) {
        ncclResult_t st = ncclSuccess;
        const ncclResult_t r = n.CommGetAsyncError(c->comm, &st);
        if (r != ncclSuccess) st = r;
        if (st == ncclSuccess) return LC_OK;
        if (st != ncclInProgress) {
            const char *msg = n.GetErrorString(st);
            abort_comm(c);
            return lc_fail(LC_ERR_CUDA, "%s: NCCL error %d (%s); communicator aborted", what, (int)st, msg);
        }
        if (Clock::now() > deadline) {
            abort_comm(c);
            return lc_fail(LC_ERR_TIMEOUT, "%s: no progress within %d ms (a rank did not arrive); communicator aborted",
                           what, c->timeout_ms);
        }
        std::this_thread::yield();
    }
}

}  // namespace

extern "C" int lc_comm_unique_id(void *id128) {
    LC_REQUIRE(id128, LC_ERR_INVALID, "lc_comm_unique_id: null out");
    int s = need_nccl("lc_comm_unique_id");
    if (s) return s;
    static_assert(sizeof(ncclUniqueId) == 128, "NCCL unique id is 128 bytes");
    ncclUniqueId id;
    const ncclResult_t r = nccl().GetUniqueId(&id);
    LC_REQUIRE(r == ncclSuccess, LC_ERR_CUDA, "ncclGetUniqueId: %s", nccl().GetErrorString(r));
    memcpy(id128, &id, sizeof(id));
    return LC_OK;
}

extern "C" int lc_comm_init(lc_ctx *ctx, const void *id128, int n_ranks, int rank, int timeout_ms, lc_comm **out) {
    LC_REQUIRE(ctx && id128 && out, LC_ERR_INVALID, "lc_comm_init: null argument");
    *out = nullptr;
    LC_REQUIRE(n_ranks >= 1 && rank >= 0 && rank < n_ranks, LC_ERR_INVALID, "lc_comm_init: rank %d of %d", rank,
               n_ranks);
    LC_REQUIRE(timeout_ms > 0, LC_ERR_INVALID, "lc_comm_init: timeout_ms must be > 0");
    int s = need_nccl("lc_comm_init");
    if (s) return s;
    if ((s = lc_use_device(ctx))) return s;
    lc_comm *c = new lc_comm();
    c->n_ranks = n_ranks, c->rank = rank, c->device = ctx->device, c->timeout_ms = timeout_ms;
    ncclUniqueId id;
    memcpy(&id, id128, sizeof(id));
    ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
    cfg.blocking = 0;  // creation and collectives return at once; the waits below are bounded
    const Clock::time_point deadline = Clock::now() + std::chrono::milliseconds(timeout_ms);
    const ncclResult_t r = nccl().CommInitRankConfig(&c->comm, n_ranks, id, rank, &cfg);
    if (r != ncclSuccess && r != ncclInProgress) {
        const char *msg = nccl().GetErrorString(r);
        if (c->comm) nccl().CommAbort(c->comm);
        delete c;
        return lc_fail(LC_ERR_CUDA, "ncclCommInitRankConfig: %s", msg);
    }
    s = wait_ready(c, deadline, "lc_comm_init");
    if (s) {
        delete c;
        return s;
    }
    *out = c;
    return LC_OK;
}

extern "C" int lc_comm_destroy(lc_comm *c) {
    if (!c) return LC_OK;
    int s = LC_OK;
    if (c->comm && !c->aborted) {
        const NcclApi &n = nccl();
        // finalize flushes outstanding work; bounded like every wait here (an
        // expired wait aborts the communicator instead)
        const Clock::time_point deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
        const ncclResult_t r = n.CommFinalize(c->comm);
        if (r == ncclSuccess || r == ncclInProgress)
            s = wait_ready(c, deadline, "lc_comm_destroy");  // aborts on expiry or error
        else
            abort_comm(c);
        if (c->comm && !c->aborted) n.CommDestroy(c->comm);
    }
    delete c;
    return s;
}

extern "C" int lc_comm_rank(const lc_comm *c, int *rank, int *n_ranks) {
    LC_REQUIRE(c, LC_ERR_INVALID, "lc_comm_rank: null comm");
    if (rank) *rank = c->rank;
    if (n_ranks) *n_ranks = c->n_ranks;
    return LC_OK;
}

extern "C" int lc_comm_allreduce_max_keys(lc_ctx *ctx, lc_comm *c, uint64_t *keys, uint32_t n) {
    LC_REQUIRE(ctx && c, LC_ERR_INVALID, "lc_comm_allreduce_max_keys: null argument");
    LC_REQUIRE(!c->aborted && c->comm, LC_ERR_INVALID, "lc_comm_allreduce_max_keys: communicator was aborted");
    LC_REQUIRE(c->device == ctx->device, LC_ERR_INVALID,
               "lc_comm_allreduce_max_keys: communicator of device %d, context of device %d", c->device, ctx->device);
    if (n == 0) return LC_OK;
    LC_REQUIRE(keys, LC_ERR_INVALID, "lc_comm_allreduce_max_keys: null keys");
    int s = lc_use_device(ctx);
    if (s) return s;
    const NcclApi &nc = nccl();
    const Clock::time_point deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    // keys compare as signed int64 (lc_pack_key)
    const ncclResult_t r = nc.AllReduce(keys, keys, n, ncclInt64, ncclMax, c->comm, ctx->stream);
    if (r != ncclSuccess && r != ncclInProgress) {
        const char *msg = nc.GetErrorString(r);
        abort_comm(c);
        return lc_fail(LC_ERR_CUDA, "ncclAllReduce: %s; communicator aborted", msg);
    }
    return wait_ready(c, deadline, "lc_comm_allreduce_max_keys");
}

extern "C" int lc_comm_wait(lc_ctx *ctx, lc_comm *c) {
    LC_REQUIRE(ctx && c, LC_ERR_INVALID, "lc_comm_wait: null argument");
    LC_REQUIRE(!c->aborted && c->comm, LC_ERR_INVALID, "lc_comm_wait: communicator was aborted");
    int s = lc_use_device(ctx);
    if (s) return s;
    const NcclApi &nc = nccl();
    const Clock::time_point deadline = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
    for (;;) {
        const cudaError_t q = cudaStreamQuery(ctx->stream);
        if (q == cudaSuccess) return LC_OK;
        if (q != cudaErrorNotReady) return lc_fail(LC_ERR_CUDA, "lc_comm_wait: %s", cudaGetErrorString(q));
        ncclResult_t st = ncclSuccess;
        nc.CommGetAsyncError(c->comm, &st);
        if (st != ncclSuccess && st != ncclInProgress) {
            const char *msg = nc.GetErrorString(st);
            abort_comm(c);
            return lc_fail(LC_ERR_CUDA, "lc_comm_wait: NCCL error %d (%s); communicator aborted", (int)st, msg);
        }
        if (Clock::now() > deadline) {
            abort_comm(c);
            // the abort ends the communicator's kernels; let the stream drain (bounded)
            const Clock::time_point drain = Clock::now() + std::chrono::milliseconds(c->timeout_ms);
            while (cudaStreamQuery(ctx->stream) == cudaErrorNotReady && Clock::now() < drain)
                std::this_thread::yield();
            return lc_fail(LC_ERR_TIMEOUT,
                           "lc_comm_wait: the reduction did not complete within %d ms (a rank did not arrive); "
                           "communicator aborted",
                           c->timeout_ms);
        }
        std::this_thread::yield();
    }
}

extern "C" int lc_lm_head_argmax_sharded(lc_ctx *ctx, lc_comm *c, int dtype, const float *x, const void *w_shard,
                                         uint32_t m, uint32_t k, uint32_t n_local, uint32_t row_offset,
                                         uint64_t *keys) {
    LC_REQUIRE(ctx && c, LC_ERR_INVALID, "lc_lm_head_argmax_sharded: null argument");
    const int sync = ctx->sync;
    ctx->sync = 0;  // the local step is enqueued; one bounded wait below covers both
    int s = lc_lm_head_argmax(ctx, dtype, x, w_shard, m, k, n_local, row_offset, keys, nullptr);
    ctx->sync = sync;
    if (s) return s;
    if ((s = lc_comm_allreduce_max_keys(ctx, c, keys, m))) return s;
    return sync ? lc_comm_wait(ctx, c) : LC_OK;
}
