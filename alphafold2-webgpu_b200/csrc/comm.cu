// comm.cu -- the pair representation sharded by rows i across the GPUs of one
// box (one process and one af2 context per GPU), with NCCL over NVLink for the
// exchange steps.  The reference has no multi-GPU code; this follows the
// partitioning its operators allow:
//
//   outgoing triangle  x[i,j] = sum_k a[i,k] b[j,k]: every rank projects its
//                      own pair rows; the projected b operand ([row][h][k],
//                      one contiguous block per rank) is all-gathered in place,
//                      and each rank contracts and finishes its own rows;
//   incoming triangle  incoming(z) = T(outgoing(T(z))) with the transposed
//                      mask, T the transpose of the pair (x[i,j] = sum_k a[k,j]
//                      b[k,i] is the outgoing product of the transposed pair):
//                      the pair and the mask are transposed across ranks by an
//                      all-to-all (pack, NCCL send/recv, unpack), the outgoing
//                      path runs on the transposed rows, and the result is
//                      transposed back.  Every operand value and every
//                      accumulation order is the one of the single-GPU path, so
//                      the sharded result is bit-identical to it.
//   transition / OPM   row-local (every output row depends on its own pair row,
//                      and on the whole MSA): no exchange.
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

// pack[s][j][i][:] = src[i][s * rows + j][:] for every destination rank s:
// the block of this rank's rows that rank s needs, already transposed.
// unit = bytes moved per thread step (16, 4 or 2).
template <typename U>
__global__ void transpose_pack_kernel(const U *__restrict__ src, U *__restrict__ pack, int rows, int n,
                                      int units_per_pair) {
  const int64_t total = static_cast<int64_t>(rows) * n * units_per_pair;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int u = static_cast<int>(idx % units_per_pair);
    const int64_t pair = idx / units_per_pair;  // destination order: (s, j, i)
    const int i = static_cast<int>(pair % rows);
    const int64_t sj = pair / rows;              // s * rows + j = the source column
    pack[idx] = src[(static_cast<int64_t>(i) * n + sj) * units_per_pair + u];
  }
}

// dst[j][r * rows + i][:] = recv[r][j][i][:]: the blocks received from every
// rank r placed at their columns.
template <typename U>
__global__ void transpose_unpack_kernel(const U *__restrict__ recv, U *__restrict__ dst, int rows, int n,
                                        int units_per_pair) {
  const int64_t total = static_cast<int64_t>(rows) * n * units_per_pair;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int u = static_cast<int>(idx % units_per_pair);
    const int64_t pair = idx / units_per_pair;  // destination order: (j, column)
    const int64_t col = pair % n;
    const int j = static_cast<int>(pair / n);
    const int r = static_cast<int>(col / rows), i = static_cast<int>(col % rows);
    dst[idx] = recv[((static_cast<int64_t>(r) * rows + j) * rows + i) * units_per_pair + u];
  }
}

template <typename U>
af2_status launch_transpose_kernels(af2_ctx *ctx, const void *src, void *pack, void *recv, void *dst, int rows, int n,
                                    size_t pair_bytes, cudaStream_t stream) {
  const int upp = static_cast<int>(pair_bytes / sizeof(U));
  const int64_t total = static_cast<int64_t>(rows) * n * upp;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 16LL * ctx->sm_count));
  {
    LaunchScope scope(ctx, stream, kProfShardTranspose);
    transpose_pack_kernel<U><<<blocks, 256, 0, stream>>>(static_cast<const U *>(src), static_cast<U *>(pack), rows, n,
                                                         upp);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(ctx, e, "transpose pack");
  // all-to-all: block s of pack goes to rank s; block r of recv comes from rank r
  const size_t block = static_cast<size_t>(rows) * rows * pair_bytes;
  ncclComm_t comm = comm_of(ctx);
  ncclResult_t r = g_nccl.GroupStart();
  for (int peer = 0; r == ncclSuccess && peer < ctx->nranks; ++peer) {
    r = g_nccl.Send(static_cast<const char *>(pack) + peer * block, block, ncclChar, peer, comm, stream);
    if (r == ncclSuccess) r = g_nccl.Recv(static_cast<char *>(recv) + peer * block, block, ncclChar, peer, comm, stream);
  }
  const ncclResult_t r2 = g_nccl.GroupEnd();
  if (r != ncclSuccess) return nccl_fail(ctx, r, "pair transpose all-to-all");
  if (r2 != ncclSuccess) return nccl_fail(ctx, r2, "pair transpose all-to-all");
  {
    LaunchScope scope(ctx, stream, kProfShardTranspose);
    transpose_unpack_kernel<U><<<blocks, 256, 0, stream>>>(static_cast<const U *>(recv), static_cast<U *>(dst), rows,
                                                           n, upp);
  }
  e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "transpose unpack");
}

}  // namespace

// The transpose of a row-sharded [n][n] pair of `pair_bytes` per pair: this
// rank holds rows [rank * rows, (rank + 1) * rows) of src and receives the
// same rows of the transpose in dst.  pack and recv hold rows * n pairs each.
af2_status shard_transpose(af2_ctx *ctx, const void *src, void *dst, void *pack, void *recv, int rows, int n,
                           size_t pair_bytes, cudaStream_t stream) {
  if (pair_bytes % 16 == 0)
    return launch_transpose_kernels<uint4>(ctx, src, pack, recv, dst, rows, n, pair_bytes, stream);
  if (pair_bytes % 4 == 0)
    return launch_transpose_kernels<uint32_t>(ctx, src, pack, recv, dst, rows, n, pair_bytes, stream);
  return launch_transpose_kernels<uint16_t>(ctx, src, pack, recv, dst, rows, n, pair_bytes, stream);
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
  if (n % R != 0 || (n / R) % 8 != 0)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "the sharded triangle needs length divisible by 8 x the rank count");
  if (direction == AF2_INCOMING && out_dtype != z_dtype)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "the sharded incoming update writes the dtype of z");
  const int64_t rows = n / R;
  const int residual = options ? options->residual : 0;
  cudaSetDevice(ctx->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const TriangleLayout L = triangle_layout(n, shape->c_z, shape->c_hidden, options ? options->block_rows : 0,
                                           z_dtype, rows);
  if ((st = ensure(ctx, ctx->workspace, L.total, "triangle scratch")) != AF2_OK) return st;
  TriangleExchange ex;
  ex.b_row0 = ctx->rank * rows;
  ex.all_gather = nccl_all_gather_in_place;
  if (direction == AF2_OUTGOING)
    return triangle_launch(ctx, AF2_OUTGOING, L, z, z_dtype, mask, packed_weights, epsilon, residual, out, out_dtype,
                           ctx->workspace.ptr, s, &ex);
  // incoming: transpose the pair and the mask across ranks, take the outgoing
  // update of the transposed rows in place, transpose back.
  const size_t zb = z_dtype == AF2_F32 ? 4 : 2;
  const size_t zbytes = (size_t)rows * n * shape->c_z * zb, mbytes = (size_t)rows * n * sizeof(float);
  const size_t off_zt = 0, off_mt = align_up(zbytes, 256), off_pack = off_mt + align_up(mbytes, 256),
               off_recv = off_pack + align_up(zbytes, 256), total = off_recv + align_up(zbytes, 256);
  if ((st = ensure(ctx, ctx->shard_scratch, total, "pair transpose scratch")) != AF2_OK) return st;
  uint8_t *sc = static_cast<uint8_t *>(ctx->shard_scratch.ptr);
  void *zt = sc + off_zt, *mt = sc + off_mt, *pack = sc + off_pack, *recv = sc + off_recv;
  if ((st = shard_transpose(ctx, z, zt, pack, recv, (int)rows, (int)n, shape->c_z * zb, s)) != AF2_OK ||
      (st = shard_transpose(ctx, mask, mt, pack, recv, (int)rows, (int)n, sizeof(float), s)) != AF2_OK ||
      (st = triangle_launch(ctx, AF2_OUTGOING, L, zt, z_dtype, static_cast<const float *>(mt), packed_weights,
                            epsilon, residual, zt, z_dtype, ctx->workspace.ptr, s, &ex)) != AF2_OK)
    return st;
  return shard_transpose(ctx, zt, out, pack, recv, (int)rows, (int)n, shape->c_z * zb, s);
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
