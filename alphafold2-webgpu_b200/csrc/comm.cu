// comm.cu -- the pair representation sharded by rows i across the GPUs of one
// box (one process and one af2 context per GPU), with NCCL over NVLink for the
// exchange steps.  The reference has no multi-GPU code; this follows the
// partitioning its operators allow:
//
// Exchanges: the triangle's all-to-alls copy straight into the peers' shard
// scratch, which every rank maps with CUDA IPC (the handles are all-gathered
// over NCCL once per allocation), with copy-engine copies on one stream per
// peer issued as soon as the kernel producing each piece has been queued (the
// projection in two halves of its rows, the contraction one destination row
// block at a time, the peers' blocks first), so the copies overlap the
// kernels; a four-byte NCCL all-reduce before the first copy (no rank writes
// into a buffer a peer may still be reading) and one after each exchange
// (every rank's data has landed before anyone reads it) order them on the
// device.  Where the mapping is refused the exchange falls back to NCCL
// send/recv after each whole kernel.
//
//   triangle (both)    every rank projects its own pair rows, split into R
//                      groups of 128 / R hidden channels; an all-to-all gives
//                      every rank its channel group of every rank's rows, so
//                      each rank contracts its channels over the whole N x N
//                      (the incoming product's k running over the ranks' row
//                      blocks in order); a second all-to-all returns all 128
//                      channels of each rank's own rows for the output
//                      projection.  Per direction a rank moves 3 (R-1)/R^2 of a
//                      projected operand; every operand value and accumulation
//                      order is the single-GPU one, so results are bit-identical.
//   outer product mean every rank holds, normalises and projects its own
//                      residue columns of the MSA; the right operand is
//                      all-gathered and each rank finishes its own rows.
//   transition         row-local: no exchange.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>
#include <type_traits>

#include "af2_device.cuh"
#include "af2_internal.h"
#include "watchdog.h"

namespace af2 {
namespace {

constexpr int64_t C_CHANNELS = 128;  // hidden channels of the padded triangle kernels

// NCCL entry points, taken from the libnccl.so.2 of the process (the one
// torch.distributed already loaded, or the system's) when a communicator is
// first created.  nccl.h supplies the types only.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId *) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*AllGather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                            cudaStream_t) = nullptr;
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t *) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  bool ok = false;
};
NcclApi g_nccl;
std::once_flag g_nccl_once;

void load_nccl() {
  void *h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_LOCAL);
  if (!h) return;
  auto sym = [&](auto &fn, const char *name) { fn = reinterpret_cast<std::remove_reference_t<decltype(fn)>>(dlsym(h, name)); };
  sym(g_nccl.GetUniqueId, "ncclGetUniqueId");
  sym(g_nccl.CommInitRank, "ncclCommInitRank");
  sym(g_nccl.CommDestroy, "ncclCommDestroy");
  sym(g_nccl.AllGather, "ncclAllGather");
  sym(g_nccl.AllReduce, "ncclAllReduce");
  sym(g_nccl.Send, "ncclSend");
  sym(g_nccl.Recv, "ncclRecv");
  sym(g_nccl.GroupStart, "ncclGroupStart");
  sym(g_nccl.GroupEnd, "ncclGroupEnd");
  sym(g_nccl.GetErrorString, "ncclGetErrorString");
  sym(g_nccl.CommGetAsyncError, "ncclCommGetAsyncError");
  sym(g_nccl.CommAbort, "ncclCommAbort");
  g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy && g_nccl.AllGather && g_nccl.AllReduce &&
              g_nccl.Send && g_nccl.Recv && g_nccl.GroupStart && g_nccl.GroupEnd && g_nccl.GetErrorString &&
              g_nccl.CommGetAsyncError && g_nccl.CommAbort;
}

bool nccl_available() {
  std::call_once(g_nccl_once, load_nccl);
  return g_nccl.ok;
}

af2_status nccl_fail(af2_ctx *ctx, ncclResult_t r, const char *what) {
  return fail(ctx, AF2_ERR_NCCL, std::string(what) + ": " + g_nccl.GetErrorString(r));
}

ncclComm_t comm_of(af2_ctx *ctx) { return static_cast<ncclComm_t>(ctx->nccl_comm); }

}  // namespace

// NCCL send/recv form of the exchange (the fallback when the peers' scratch cannot be mapped).
static af2_status nccl_exchange(af2_ctx *ctx, const ShardTransfer *tr, int count, cudaStream_t stream) {
  ncclComm_t comm = comm_of(ctx);
  ncclResult_t r = g_nccl.GroupStart();
  for (int k = 0; r == ncclSuccess && k < count; ++k) {
    const char *src = static_cast<const char *>(tr[k].send);
    char *dst = static_cast<char *>(tr[k].recv);
    for (int peer = 0; r == ncclSuccess && peer < ctx->nranks; ++peer) {
      if (peer == ctx->rank) continue;
      r = g_nccl.Send(src + peer * tr[k].stride, tr[k].bytes, ncclChar, peer, comm, stream);
      if (r == ncclSuccess) r = g_nccl.Recv(dst + peer * tr[k].stride, tr[k].bytes, ncclChar, peer, comm, stream);
    }
  }
  const ncclResult_t r2 = g_nccl.GroupEnd();
  if (r != ncclSuccess) return nccl_fail(ctx, r, "channel all-to-all");
  if (r2 != ncclSuccess) return nccl_fail(ctx, r2, "channel all-to-all");
  return AF2_OK;
}

// Every rank's stream reaches this point before any continues (a four-byte all-reduce).
static af2_status device_barrier(af2_ctx *ctx, cudaStream_t stream) {
  const ncclResult_t r = g_nccl.AllReduce(ctx->sync_word, ctx->sync_word, 1, ncclInt32, ncclSum, comm_of(ctx), stream);
  return r == ncclSuccess ? AF2_OK : nccl_fail(ctx, r, "exchange barrier");
}

static void close_peers(af2_ctx *ctx) {
  for (void *&p : ctx->peer_scratch)
    if (p) {
      cudaIpcCloseMemHandle(p);
      p = nullptr;
    }
  ctx->peer_of = nullptr;
}

// Maps every peer's shard scratch (a collective: all ranks call it with their own allocation).
static af2_status map_peers(af2_ctx *ctx, cudaStream_t stream) {
  close_peers(ctx);
  const int R = ctx->nranks;
  cudaIpcMemHandle_t mine;
  std::memset(&mine, 0, sizeof mine);
  int ok = cudaIpcGetMemHandle(&mine, ctx->shard_scratch.ptr) == cudaSuccess ? 1 : 0;
  if (!ok) cudaGetLastError();
  // [R][handle + flag], gathered through device memory
  const size_t rec = sizeof(cudaIpcMemHandle_t) + 16;
  std::vector<char> host(rec * R, 0);
  std::memcpy(host.data() + rec * ctx->rank, &mine, sizeof mine);
  std::memcpy(host.data() + rec * ctx->rank + sizeof mine, &ok, sizeof ok);
  char *dev = nullptr;
  if (cudaMalloc(&dev, rec * R) != cudaSuccess) return cuda_fail(ctx, cudaGetLastError(), "handle exchange buffer");
  cudaError_t e = cudaMemcpyAsync(dev + rec * ctx->rank, host.data() + rec * ctx->rank, rec, cudaMemcpyHostToDevice,
                                  stream);
  ncclResult_t r = e == cudaSuccess ? g_nccl.AllGather(dev + rec * ctx->rank, dev, rec, ncclChar, comm_of(ctx), stream)
                                    : ncclSuccess;
  if (e == cudaSuccess && r == ncclSuccess)
    e = cudaMemcpyAsync(host.data(), dev, rec * R, cudaMemcpyDeviceToHost, stream);
  af2_status waited = e == cudaSuccess && r == ncclSuccess ? comm_wait(ctx, stream, "handle exchange") : AF2_OK;
  cudaFree(dev);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "all-gather of the scratch handles");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "handle exchange");
  if (waited != AF2_OK) return waited;
  bool all = true;
  for (int p = 0; p < R; ++p) {
    int flag = 0;
    std::memcpy(&flag, host.data() + rec * p + sizeof mine, sizeof flag);
    all = all && flag;
  }
  ctx->peer_scratch.assign(R, nullptr);
  for (int p = 0; all && p < R; ++p) {
    if (p == ctx->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, host.data() + rec * p, sizeof h);
    if (cudaIpcOpenMemHandle(&ctx->peer_scratch[p], h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ctx->peer_scratch[p] = nullptr;
      all = false;
    }
  }
  // every rank learns whether all mappings succeeded, so all take the same path
  int fail_count = all ? 0 : 1;
  int *dflag = nullptr;
  if (cudaMalloc(&dflag, sizeof(int)) != cudaSuccess) return cuda_fail(ctx, cudaGetLastError(), "mapping vote");
  e = cudaMemcpyAsync(dflag, &fail_count, sizeof(int), cudaMemcpyHostToDevice, stream);
  r = e == cudaSuccess ? g_nccl.AllReduce(dflag, dflag, 1, ncclInt32, ncclSum, comm_of(ctx), stream) : ncclSuccess;
  if (e == cudaSuccess && r == ncclSuccess) e = cudaMemcpyAsync(&fail_count, dflag, sizeof(int), cudaMemcpyDeviceToHost, stream);
  waited = e == cudaSuccess && r == ncclSuccess ? comm_wait(ctx, stream, "mapping vote") : AF2_OK;
  cudaFree(dflag);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "mapping vote");
  if (e != cudaSuccess) return cuda_fail(ctx, e, "mapping vote");
  if (waited != AF2_OK) return waited;
  if (fail_count > 0) {
    close_peers(ctx);
    ctx->ipc_failed = true;
    return AF2_OK;
  }
  ctx->peer_of = ctx->shard_scratch.ptr;
  return AF2_OK;
}

// Direct exchange: whether copies can go straight into the peers' scratch (mapping it first).
static bool ipc_direct(af2_ctx *ctx, cudaStream_t stream, af2_status *status) {
  *status = AF2_OK;
  if (ctx->ipc_failed || !ctx->shard_scratch.ptr) return false;
  if (ctx->peer_of != ctx->shard_scratch.ptr && (*status = map_peers(ctx, stream)) != AF2_OK) return false;
  return !ctx->ipc_failed && ctx->peer_of == ctx->shard_scratch.ptr;
}

static af2_status ipc_open(af2_ctx *ctx, cudaStream_t stream) { return device_barrier(ctx, stream); }

static void *ipc_peer_base(af2_ctx *ctx, int peer) {
  return (peer >= 0 && peer < static_cast<int>(ctx->peer_scratch.size())) ? ctx->peer_scratch[peer] : nullptr;
}

// One copy on the peer's copy stream, after everything queued on `stream` so far.
static af2_status ipc_send(af2_ctx *ctx, const void *src, const void *dst_local, size_t bytes, int peer,
                           cudaStream_t stream) {
  const char *base = static_cast<const char *>(ctx->shard_scratch.ptr), *dst = static_cast<const char *>(dst_local);
  if (peer < 0 || peer >= ctx->nranks || peer == ctx->rank || dst < base ||
      dst + bytes > base + ctx->shard_scratch.bytes || !ctx->peer_scratch[peer])
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "exchange copy outside the shard scratch");
  cudaEvent_t fork = ctx->copy_events[ctx->rank];
  cudaStream_t cs = ctx->copy_streams[peer];
  cudaError_t e = cudaEventRecord(fork, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(cs, fork, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(static_cast<char *>(ctx->peer_scratch[peer]) + (dst - base), src, bytes,
                        cudaMemcpyDeviceToDevice, cs);
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "exchange copy");
}

// Joins the copy streams into `stream`, then the barrier after which every rank's data has landed.
static af2_status ipc_close(af2_ctx *ctx, cudaStream_t stream) {
  cudaError_t e = cudaSuccess;
  for (int p = 0; e == cudaSuccess && p < ctx->nranks; ++p) {
    if (p == ctx->rank) continue;
    e = cudaEventRecord(ctx->copy_events[p], ctx->copy_streams[p]);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ctx->copy_events[p], 0);
  }
  if (e != cudaSuccess) return cuda_fail(ctx, e, "exchange join");
  return device_barrier(ctx, stream);
}

static af2_status nccl_all_gather_in_place(af2_ctx *ctx, void *full, size_t bytes_per_rank, cudaStream_t stream) {
  const ncclResult_t r =
      g_nccl.AllGather(static_cast<const char *>(full) + static_cast<size_t>(ctx->rank) * bytes_per_rank, full,
                    bytes_per_rank, ncclChar, comm_of(ctx), stream);
  return r == ncclSuccess ? AF2_OK : nccl_fail(ctx, r, "all-gather of the projected b operand");
}

void comm_destroy(af2_ctx *ctx) {
  close_peers(ctx);
  for (cudaStream_t cs : ctx->copy_streams)
    if (cs) cudaStreamDestroy(cs);
  for (cudaEvent_t ev : ctx->copy_events)
    if (ev) cudaEventDestroy(ev);
  ctx->copy_streams.clear();
  ctx->copy_events.clear();
  ctx->peer_scratch.clear();
  if (ctx->sync_word) {
    cudaFree(ctx->sync_word);
    ctx->sync_word = nullptr;
  }
  ctx->ipc_failed = false;
  ctx->comm_aborted = false;
  if (ctx->nccl_comm) {
    g_nccl.CommDestroy(comm_of(ctx));
    ctx->nccl_comm = nullptr;
  }
  if (ctx->shard_scratch.ptr) {
    cudaFree(ctx->shard_scratch.ptr);
    ctx->allocated -= ctx->shard_scratch.bytes;
    ctx->shard_scratch = DeviceBuffer{};
  }
  ctx->nranks = 1;
  ctx->rank = 0;
}

// Ends the communicator after a failure: its kernels stop waiting, so the streams drain.
static void comm_abort(af2_ctx *ctx) {
  if (!ctx->nccl_comm) return;
  g_nccl.CommAbort(comm_of(ctx));
  ctx->nccl_comm = nullptr;
  ctx->comm_aborted = true;
}

static af2_status comm_ready(af2_ctx *ctx) {
  if (ctx->comm_aborted)
    return fail(ctx, AF2_ERR_NCCL,
                "the communicator was aborted after a failure: af2_comm_destroy, then af2_comm_init");
  if (!ctx->nccl_comm) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "af2_comm_init has not been called on this context");
  return AF2_OK;
}

af2_status comm_wait(af2_ctx *ctx, cudaStream_t stream, const char *what) {
  if (!ctx->nccl_comm) {
    const cudaError_t e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, what);
  }
  cudaError_t stream_error = cudaSuccess;
  ncclResult_t peer_error = ncclSuccess;
  ncclComm_t comm = comm_of(ctx);
  const WaitOutcome w = wait_with_watchdog(
      [&] {
        const cudaError_t e = cudaStreamQuery(stream);
        if (e == cudaSuccess) return StreamState::kDone;
        if (e == cudaErrorNotReady) return StreamState::kPending;
        stream_error = e;
        return StreamState::kError;
      },
      [&] {
        ncclResult_t r = ncclSuccess;
        if (g_nccl.CommGetAsyncError(comm, &r) != ncclSuccess) r = ncclInternalError;
        if (r == ncclSuccess || r == ncclInProgress) return PeerState::kOk;
        peer_error = r;
        return PeerState::kError;
      },
      ctx->comm_timeout_s);
  if (w == WaitOutcome::kDone) return AF2_OK;
  if (w == WaitOutcome::kStreamError) return cuda_fail(ctx, stream_error, what);
  std::string message = std::string(what) + ": " + wait_outcome_text(w);
  if (w == WaitOutcome::kPeerError) message += std::string(" (") + g_nccl.GetErrorString(peer_error) + ")";
  else message += " (" + std::to_string(ctx->comm_timeout_s) + " s)";
  comm_abort(ctx);
  // the aborted communicator's kernels return; give the stream a bounded time to drain
  const WaitOutcome drained = wait_with_watchdog(
      [&] {
        const cudaError_t e = cudaStreamQuery(stream);
        return e == cudaSuccess ? StreamState::kDone : e == cudaErrorNotReady ? StreamState::kPending : StreamState::kError;
      },
      [] { return PeerState::kOk; }, 30.0);
  if (drained != WaitOutcome::kDone) message += "; the stream had not drained 30 s after the abort";
  return fail(ctx, AF2_ERR_NCCL, message + "; the communicator was aborted: af2_comm_destroy, then af2_comm_init");
}

}  // namespace af2

using namespace af2;

extern "C" {

af2_status af2_comm_unique_id(void *unique_id) {
  if (!unique_id) return AF2_ERR_INVALID_ARGUMENT;
  if (!nccl_available()) return AF2_ERR_NCCL;
  ncclUniqueId id;
  if (g_nccl.GetUniqueId(&id) != ncclSuccess) return AF2_ERR_NCCL;
  std::memcpy(unique_id, &id, sizeof id);
  return AF2_OK;
}

af2_status af2_comm_init(af2_ctx *ctx, const void *unique_id, int nranks, int rank) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (!unique_id || nranks < 1 || rank < 0 || rank >= nranks)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a unique id, nranks >= 1 and 0 <= rank < nranks are required");
  if (ctx->nccl_comm || ctx->comm_aborted)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "this context already has a communicator (af2_comm_destroy first)");
  if (!nccl_available()) return fail(ctx, AF2_ERR_NCCL, "libnccl.so.2 could not be opened");
  cudaSetDevice(ctx->device);
  ncclUniqueId id;
  std::memcpy(&id, unique_id, sizeof id);
  ncclComm_t comm = nullptr;
  const ncclResult_t r = g_nccl.CommInitRank(&comm, nranks, id, rank);
  if (r != ncclSuccess) return nccl_fail(ctx, r, "ncclCommInitRank");
  ctx->nccl_comm = comm;
  ctx->nranks = nranks;
  ctx->rank = rank;
  // exchange resources: a barrier word, one copy stream and event per rank
  cudaError_t e = cudaMalloc(&ctx->sync_word, 256);
  if (e == cudaSuccess) e = cudaMemset(ctx->sync_word, 0, 256);
  ctx->copy_streams.assign(nranks, nullptr);
  ctx->copy_events.assign(nranks, nullptr);
  for (int p = 0; e == cudaSuccess && p < nranks; ++p) {
    e = cudaStreamCreateWithFlags(&ctx->copy_streams[p], cudaStreamNonBlocking);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->copy_events[p], cudaEventDisableTiming);
  }
  if (e != cudaSuccess) {
    comm_destroy(ctx);
    return cuda_fail(ctx, e, "exchange streams");
  }
  return AF2_OK;
}

af2_status af2_comm_destroy(af2_ctx *ctx) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  // a failed wait aborts the communicator; the rest of the teardown is local
  af2_status st = ctx->stream ? comm_wait(ctx, ctx->stream, "af2_comm_destroy") : AF2_OK;
  if (ctx->nccl_comm && ctx->peer_of) {
    // every rank closes its mappings of the peers' scratch before any rank frees its own
    close_peers(ctx);
    if (st == AF2_OK && (st = device_barrier(ctx, ctx->stream)) == AF2_OK)
      st = comm_wait(ctx, ctx->stream, "af2_comm_destroy");
  }
  comm_destroy(ctx);
  return st;
}

af2_status af2_comm_abort(af2_ctx *ctx) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  comm_abort(ctx);
  // the streams hold no collective that can still wait: drain them (bounded) before freeing
  af2_status st = AF2_OK;
  if (ctx->stream) {
    const WaitOutcome w = wait_with_watchdog(
        [&] {
          const cudaError_t e = cudaStreamQuery(ctx->stream);
          return e == cudaSuccess ? StreamState::kDone : e == cudaErrorNotReady ? StreamState::kPending
                                                                                : StreamState::kError;
        },
        [] { return PeerState::kOk; }, 30.0);
    if (w != WaitOutcome::kDone) st = fail(ctx, AF2_ERR_NCCL, "af2_comm_abort: the stream did not drain");
  }
  comm_destroy(ctx);
  return st;
}

af2_status af2_triangle_multiplication_sharded(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                               const void *z, int z_dtype, const float *mask,
                                               const float *packed_weights, int64_t weight_count, double epsilon,
                                               const af2_triangle_options *options, void *out, int out_dtype,
                                               void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  char message[256];
  af2_status st = af2_triangle_check(direction, shape, weight_count, epsilon, message, sizeof message);
  if (st != AF2_OK) return fail(ctx, st, message);
  if ((st = comm_ready(ctx)) != AF2_OK) return st;
  if (!z || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  const bool dtypes_ok = (z_dtype == AF2_F32 || z_dtype == AF2_F16 || z_dtype == AF2_BF16) &&
                         (out_dtype == AF2_F32 || out_dtype == AF2_F16 || out_dtype == AF2_BF16);
  if (!dtypes_ok) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  const int64_t n = shape->length, R = ctx->nranks;
  if (C_CHANNELS % R != 0 || n % R != 0 || (n / R) % 64 != 0)
    return fail(ctx, AF2_ERR_UNSUPPORTED,
                "the sharded triangle needs a rank count dividing 128 and length divisible by 64 x the rank count");
  const int64_t rows = n / R;
  const int residual = options ? options->residual : 0;
  cudaSetDevice(ctx->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const TriangleLayout L = triangle_layout(n, shape->c_z, shape->c_hidden, 0, z_dtype, rows, direction);
  // sized for both directions at once, so the allocation the peers have mapped does not move
  // between an outgoing and an incoming call
  const TriangleLayout L2 = triangle_layout(n, shape->c_z, shape->c_hidden, 0, z_dtype, rows, 1 - direction);
  const size_t need = std::max(L.total, L2.total);
  if (ctx->shard_scratch.bytes < need && ctx->peer_of) {
    // every rank grows at the same call: all close their mappings before any frees its allocation
    close_peers(ctx);
    if ((st = device_barrier(ctx, s)) != AF2_OK) return st;
    if ((st = comm_wait(ctx, s, "scratch regrowth")) != AF2_OK) return st;
  }
  if ((st = ensure(ctx, ctx->shard_scratch, need, "sharded triangle scratch")) != AF2_OK) return st;
  TriangleShard sh;
  sh.ranks = static_cast<int>(R);
  sh.rank = ctx->rank;
  sh.exchange = nccl_exchange;
  sh.direct = ipc_direct;
  sh.open = ipc_open;
  sh.send = ipc_send;
  sh.close = ipc_close;
  sh.peer_base = ipc_peer_base;
  return triangle_launch(ctx, direction, L, z, z_dtype, mask, packed_weights, epsilon, residual, out, out_dtype,
                         ctx->shard_scratch.ptr, s, &sh);
}

af2_status af2_outer_product_mean_sharded(af2_ctx *ctx, const af2_opm_shape *shape, const void *m, int m_dtype,
                                          const float *mask, const float *packed_weights, int64_t weight_count,
                                          const af2_opm_options *options, void *out, int out_dtype, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  char message[256];
  af2_status st = af2_opm_check(shape, weight_count, message, sizeof message);
  if (st != AF2_OK) return fail(ctx, st, message);
  if ((st = comm_ready(ctx)) != AF2_OK) return st;
  if (!m || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  const bool dtypes_ok = (m_dtype == AF2_F32 || m_dtype == AF2_F16 || m_dtype == AF2_BF16) &&
                         (out_dtype == AF2_F32 || out_dtype == AF2_F16 || out_dtype == AF2_BF16);
  if (!dtypes_ok) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  const int64_t n = shape->length, R = ctx->nranks;
  if (n % R != 0 || (n / R) % 8 != 0)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "the sharded OPM needs length divisible by 8 x the rank count");
  const double ln_eps = (options && options->layer_norm_epsilon != 0) ? options->layer_norm_epsilon : 1e-5;
  const double norm_eps = (options && options->normalization_epsilon != 0) ? options->normalization_epsilon : 1e-3;
  if (!(ln_eps > 0) || !std::isfinite(ln_eps) || !(norm_eps > 0) || !std::isfinite(norm_eps))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "epsilons must be finite and positive");
  const int64_t rows = n / R;
  cudaSetDevice(ctx->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const OpmLayout L = opm_layout(shape->sequences, n, shape->c_m, shape->c_outer, shape->c_z,
                                 options ? options->row_block_residues : 0, rows, ctx->rank * rows);
  if ((st = ensure(ctx, ctx->workspace, L.total, "outer product mean scratch")) != AF2_OK) return st;
  OpmExchange ex;
  ex.rank = ctx->rank;
  ex.m_local = true;
  ex.all_gather = nccl_all_gather_in_place;
  return opm_launch(ctx, L, m, m_dtype, mask, packed_weights, ln_eps, norm_eps, options ? options->residual : 0, out,
                    out_dtype, ctx->workspace.ptr, s, &ex);
}

}  // extern "C"
