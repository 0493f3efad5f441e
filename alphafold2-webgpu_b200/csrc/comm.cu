// comm.cu -- the pair representation sharded by rows i across the GPUs of one
// box (one process and one af2 context per GPU), with NCCL over NVLink for the
// exchange steps.  The reference has no multi-GPU code; this follows the
// partitioning its operators allow:
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
//   outer product mean every rank normalises and projects its own residue
//                      columns of the (replicated) MSA; the right operand is
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
  ncclResult_t (*Send)(const void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void *, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char *(*GetErrorString)(ncclResult_t) = nullptr;
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
  sym(g_nccl.Send, "ncclSend");
  sym(g_nccl.Recv, "ncclRecv");
  sym(g_nccl.GroupStart, "ncclGroupStart");
  sym(g_nccl.GroupEnd, "ncclGroupEnd");
  sym(g_nccl.GetErrorString, "ncclGetErrorString");
  g_nccl.ok = g_nccl.GetUniqueId && g_nccl.CommInitRank && g_nccl.CommDestroy && g_nccl.AllGather && g_nccl.Send &&
              g_nccl.Recv && g_nccl.GroupStart && g_nccl.GroupEnd && g_nccl.GetErrorString;
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

// Block p of `send` to rank p, rank p's block into block p of `recv` (blocks
// `stride` bytes apart, `bytes` each).  This rank's own block is not moved: the
// triangle kernels read and write it in place.
static af2_status nccl_all_to_all(af2_ctx *ctx, const void *send, void *recv, size_t stride, size_t bytes,
                                  cudaStream_t stream) {
  const char *src = static_cast<const char *>(send);
  char *dst = static_cast<char *>(recv);
  ncclComm_t comm = comm_of(ctx);
  ncclResult_t r = g_nccl.GroupStart();
  for (int peer = 0; r == ncclSuccess && peer < ctx->nranks; ++peer) {
    if (peer == ctx->rank) continue;
    r = g_nccl.Send(src + peer * stride, bytes, ncclChar, peer, comm, stream);
    if (r == ncclSuccess) r = g_nccl.Recv(dst + peer * stride, bytes, ncclChar, peer, comm, stream);
  }
  const ncclResult_t r2 = g_nccl.GroupEnd();
  if (r != ncclSuccess) return nccl_fail(ctx, r, "channel all-to-all");
  if (r2 != ncclSuccess) return nccl_fail(ctx, r2, "channel all-to-all");
  return AF2_OK;
}

static af2_status nccl_all_gather_in_place(af2_ctx *ctx, void *full, size_t bytes_per_rank, cudaStream_t stream) {
  const ncclResult_t r =
      g_nccl.AllGather(static_cast<const char *>(full) + static_cast<size_t>(ctx->rank) * bytes_per_rank, full,
                    bytes_per_rank, ncclChar, comm_of(ctx), stream);
  return r == ncclSuccess ? AF2_OK : nccl_fail(ctx, r, "all-gather of the projected b operand");
}

void comm_destroy(af2_ctx *ctx) {
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
  if (ctx->nccl_comm) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "this context already has a communicator");
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
  return AF2_OK;
}

af2_status af2_comm_destroy(af2_ctx *ctx) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  comm_destroy(ctx);
  return AF2_OK;
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
  if (!ctx->nccl_comm) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "af2_comm_init has not been called on this context");
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
  if ((st = ensure(ctx, ctx->shard_scratch, L.total, "sharded triangle scratch")) != AF2_OK) return st;
  TriangleShard sh;
  sh.ranks = static_cast<int>(R);
  sh.rank = ctx->rank;
  sh.all_to_all = nccl_all_to_all;
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
  if (!ctx->nccl_comm) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "af2_comm_init has not been called on this context");
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
  ex.all_gather = nccl_all_gather_in_place;
  return opm_launch(ctx, L, m, m_dtype, mask, packed_weights, ln_eps, norm_eps, options ? options->residual : 0, out,
                    out_dtype, ctx->workspace.ptr, s, &ex);
}

}  // extern "C"
