// api.cu -- the extern "C" surface of libaf2cuda.so: contexts, validation
// that mirrors the reference's RangeError checks, the host form (upload, run,
// read back) and the device form of each operator.
#include <cudaTypedefs.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>

#include "af2_internal.h"

namespace af2 {

af2_status fail(af2_ctx *ctx, af2_status status, const std::string &message) {
  if (ctx) ctx->last_error = message;
  return status;
}

int tuning_override(const char *name, int fallback) {
  const char *v = std::getenv(name);
  if (!v || !*v) return fallback;
  char *end = nullptr;
  const long x = std::strtol(v, &end, 10);
  return (end && *end == '\0') ? static_cast<int>(x) : fallback;
}

af2_status cuda_fail(af2_ctx *ctx, cudaError_t e, const char *what) {
  const af2_status s = (e == cudaErrorMemoryAllocation) ? AF2_ERR_OUT_OF_MEMORY : AF2_ERR_CUDA;
  return fail(ctx, s, std::string(what) + ": " + cudaGetErrorString(e));
}

af2_status ensure(af2_ctx *ctx, DeviceBuffer &buf, size_t bytes, const char *what) {
  if (buf.bytes >= bytes) return AF2_OK;
  if (buf.ptr) {
    if (af2_status st = comm_wait(ctx, ctx->stream, "synchronize before regrowing scratch"); st != AF2_OK) return st;
    cudaFree(buf.ptr);
    ctx->allocated -= buf.bytes;
    buf.ptr = nullptr;
    buf.bytes = 0;
  }
  const size_t want = align_up(bytes, 1 << 20);
  cudaError_t e = cudaMalloc(&buf.ptr, want);
  if (e != cudaSuccess) {
    buf.ptr = nullptr;
    cudaGetLastError();
    return fail(ctx, AF2_ERR_OUT_OF_MEMORY,
                std::string("device allocation of ") + std::to_string(want) + " bytes for " + what + " failed: " +
                    cudaGetErrorString(e));
  }
  buf.bytes = want;
  ctx->allocated += want;
  if (ctx->allocated > ctx->peak) ctx->peak = ctx->allocated;
  return AF2_OK;
}

bool WeightKey::operator==(const WeightKey &o) const {
  if (kind != o.kind) return false;
  for (int i = 0; i < 32; ++i)
    if (ptr[i] != o.ptr[i]) return false;
  for (int i = 0; i < 8; ++i)
    if (dim[i] != o.dim[i]) return false;
  return true;
}

af2_status prepared_region(af2_ctx *ctx, const WeightKey &key, size_t bytes, void *workspace, bool allow,
                           PreparedRegion *out) {
  if (!ctx->weight_cache || !allow) {
    out->base = static_cast<uint8_t *>(workspace);
    out->fresh = true;
    return AF2_OK;
  }
  for (CachedWeights &c : ctx->cached_weights)
    if (c.key == key && c.buf.bytes >= bytes) {
      out->base = static_cast<uint8_t *>(c.buf.ptr);
      out->fresh = false;
      return AF2_OK;
    }
  CachedWeights entry;
  entry.key = key;
  const size_t want = align_up(bytes, 256);
  cudaError_t e = cudaMalloc(&entry.buf.ptr, want);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(ctx, AF2_ERR_OUT_OF_MEMORY, "device allocation for the prepared-weights cache failed");
  }
  entry.buf.bytes = want;
  ctx->allocated += want;
  if (ctx->allocated > ctx->peak) ctx->peak = ctx->allocated;
  ctx->cached_weights.push_back(entry);
  out->base = static_cast<uint8_t *>(entry.buf.ptr);
  out->fresh = true;
  return AF2_OK;
}

void clear_weight_cache(af2_ctx *ctx) {
  if (!ctx->cached_weights.empty()) cudaDeviceSynchronize();  // no kernel may still read them
  for (CachedWeights &c : ctx->cached_weights) {
    cudaFree(c.buf.ptr);
    ctx->allocated -= c.buf.bytes;
  }
  ctx->cached_weights.clear();
}

const char *profile_name(int id) {
  static const char *names[kProfCount] = {
      "triangle.prepare",    "triangle.relayout",    "triangle.project",  "triangle.contract",
      "triangle.output",     "transition.prepare",   "transition.normalize", "transition.fused",
      "q8.decode",           "weights.prepare",      "activations.convert",  "linear",
      "opm.normalize",       "opm.project",          "opm.count",         "opm.outer",
      "opm.output",          "opm.fused",            "transition.linear",
      "attention.normalize", "attention.project",    "attention.flash",   "attention.output"};
  return (id >= 0 && id < kProfCount) ? names[id] : nullptr;
}

static cudaEvent_t take_event(af2_ctx *ctx) {
  if (!ctx->free_events.empty()) {
    cudaEvent_t e = ctx->free_events.back();
    ctx->free_events.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

LaunchScope::LaunchScope(af2_ctx *ctx, cudaStream_t stream, int id) : ctx_(ctx), stream_(stream), id_(id) {
  ctx_->launches++;
  if (ctx_->profiling) {
    start_ = take_event(ctx_);
    if (start_) cudaEventRecord(start_, stream_);
  }
}

LaunchScope::~LaunchScope() {
  if (!start_) return;
  cudaEvent_t stop = take_event(ctx_);
  if (!stop) {
    ctx_->free_events.push_back(start_);
    return;
  }
  cudaEventRecord(stop, stream_);
  ctx_->pending.push_back({id_, start_, stop});
}

namespace {
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
  void *fn = nullptr;
  cudaDriverEntryPointQueryResult q{};
  if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000, cudaEnableDefault, &q) ==
          cudaSuccess &&
      q == cudaDriverEntryPointSuccess)
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
}
}  // namespace

bool encode_map_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                   uint32_t b2, CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return false;
  const cuuint64_t dims[3] = {d0, d1, d2};
  const cuuint64_t strides[2] = {stride1_bytes, stride2_bytes};
  const cuuint32_t box[3] = {b0, b1, b2};
  const cuuint32_t estr[3] = {1, 1, 1};
  return g_encode(map, dtype, 3, const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool encode_map_4d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, const uint64_t (&dims)[4],
                   const uint64_t (&strides_bytes)[3], const uint32_t (&box)[4], CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, load_encode);
  if (!g_encode) return false;
  const cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  const cuuint64_t st[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  const cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  return g_encode(map, dtype, 4, const_cast<void *>(base), d, st, b, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

constexpr int64_t kMaxSafeInteger = 9007199254740991LL;  // Number.MAX_SAFE_INTEGER

bool positive_safe(int64_t v) { return v > 0 && v <= kMaxSafeInteger; }

size_t dtype_bytes(int dtype) { return dtype == AF2_F32 ? 4 : 2; }

bool valid_dtype(int dtype) { return dtype == AF2_F32 || dtype == AF2_F16 || dtype == AF2_BF16; }

// validateTriangleInput (src/triangle/types.ts:54-89), for what a C caller hands over.
af2_status validate_triangle(af2_ctx *ctx, int direction, const af2_triangle_shape *shape, int64_t weight_count,
                             double epsilon) {
  if (!shape) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape is NULL");
  if (direction != AF2_OUTGOING && direction != AF2_INCOMING)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "direction must be 0 (outgoing) or 1 (incoming)");
  const char *names[3] = {"length", "cZ", "cHidden"};
  const int64_t vals[3] = {shape->length, shape->c_z, shape->c_hidden};
  for (int i = 0; i < 3; ++i)
    if (!positive_safe(vals[i]))
      return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string(names[i]) + " must be a positive safe integer; received " +
                                                     std::to_string(vals[i]));
  const double pair_count = (double)shape->length * (double)shape->length;
  if (pair_count * (double)std::max(shape->c_z, shape->c_hidden) > (double)kMaxSafeInteger)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "tensor dimensions exceed JavaScript's safe integer range");
  const int64_t expected = af2_triangle_weight_count(shape->c_z, shape->c_hidden);
  if (weight_count != expected)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "packed weights have " + std::to_string(weight_count) +
                                                   " values; expected " + std::to_string(expected));
  if (!(epsilon > 0) || !std::isfinite(epsilon))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "epsilon must be finite and positive; received " +
                                                   std::to_string(epsilon));
  if (shape->c_z > 128 || shape->c_hidden > 128)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "c_z and c_hidden above 128 are not supported by the sm_100a kernels");
  if (shape->length > (1 << 20))
    return fail(ctx, AF2_ERR_UNSUPPORTED, "length above 1048576 is not supported");
  return AF2_OK;
}

af2_status check_device_errors(af2_ctx *ctx) {
  unsigned int word = 0;
  cudaError_t e = cudaMemcpy(&word, ctx->err_word, sizeof(word), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "read the device error word");
  if (word != 0) {
    cudaMemset(ctx->err_word, 0, sizeof(unsigned int));
    char buf[160];
    std::snprintf(buf, sizeof buf,
                  "a kernel's bounded wait ran out (error bits 0x%x); the kernel returned without finishing", word);
    return fail(ctx, AF2_ERR_DEVICE_TIMEOUT, buf);
  }
  return AF2_OK;
}

// validate (src/evoformer/transition.ts:140-156) for a C caller, then the kernels' limits.
af2_status validate_transition(af2_ctx *ctx, const af2_transition_shape *shape, double epsilon) {
  if (!shape) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape is NULL");
  if (!positive_safe(shape->rows) || !positive_safe(shape->channels) || !positive_safe(shape->hidden_channels))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "transition dimensions must be positive safe integers");
  if ((double)shape->rows * (double)std::max(shape->channels, shape->hidden_channels) > (double)kMaxSafeInteger)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "tensor dimensions exceed JavaScript's safe integer range");
  if (!(epsilon > 0) || !std::isfinite(epsilon))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "epsilon must be finite and positive; received " +
                                                   std::to_string(epsilon));
  if (shape->channels > 4096)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "transition channels above 4096 are not supported");
  if (shape->hidden_channels > 16384)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "transition hidden channels above 16384 are not supported");
  if (shape->rows > (int64_t(1) << 30))
    return fail(ctx, AF2_ERR_UNSUPPORTED, "transition rows beyond 2^30 are not supported");
  return AF2_OK;
}

// validate (src/evoformer/outer-product-mean.ts:45-65) for a C caller, then the kernels' limits.
af2_status validate_opm(af2_ctx *ctx, const af2_opm_shape *shape, int64_t weight_count) {
  if (!shape) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape is NULL");
  const int64_t dims[5] = {shape->sequences, shape->length, shape->c_m, shape->c_outer, shape->c_z};
  for (int64_t d : dims)
    if (!positive_safe(d))
      return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "outer product mean dimensions must be positive safe integers");
  if ((double)shape->sequences * (double)shape->length * (double)shape->c_m > (double)kMaxSafeInteger ||
      (double)shape->length * (double)shape->length * (double)shape->c_z > (double)kMaxSafeInteger)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "tensor dimensions exceed JavaScript's safe integer range");
  const int64_t expected = af2_opm_weight_count(shape);
  if (weight_count != expected)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "packed weights have " + std::to_string(weight_count) +
                                                   " values; expected " + std::to_string(expected));
  if (shape->c_outer != 32)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "the sm_100a outer-product kernel is built for c_outer = 32");
  if (shape->c_m > 256) return fail(ctx, AF2_ERR_UNSUPPORTED, "c_m above 256 is not supported");
  if (shape->c_z > 4096) return fail(ctx, AF2_ERR_UNSUPPORTED, "c_z above 4096 is not supported");
  if (shape->length > 65536 || shape->sequences > (1 << 24))
    return fail(ctx, AF2_ERR_UNSUPPORTED, "length above 65536 or more than 2^24 sequences are not supported");
  return AF2_OK;
}

af2_status validate_matrix(af2_ctx *ctx, const af2_matrix &m, const char *name) {
  if (!m.values) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string(name) + " values are NULL");
  if (m.format == AF2_WEIGHTS_F32) return AF2_OK;
  if (m.format != AF2_WEIGHTS_Q8_BLOCK && m.format != AF2_WEIGHTS_Q8_CHANNEL)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string(name) + " has an unknown weight format");
  if (!m.scales) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string(name) + " scales are NULL");
  if (m.format == AF2_WEIGHTS_Q8_BLOCK && m.block <= 0)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string(name) + " block must be positive");
  return AF2_OK;
}

}  // namespace
}  // namespace af2

using namespace af2;

extern "C" {

int af2_version(void) { return AF2CUDA_VERSION; }

const char *af2_status_string(af2_status status) {
  switch (status) {
    case AF2_OK: return "ok";
    case AF2_ERR_INVALID_ARGUMENT: return "invalid argument";
    case AF2_ERR_UNSUPPORTED: return "unsupported";
    case AF2_ERR_OUT_OF_MEMORY: return "out of device memory";
    case AF2_ERR_CUDA: return "CUDA error";
    case AF2_ERR_DEVICE_TIMEOUT: return "device-side wait timed out";
    case AF2_ERR_NCCL: return "NCCL error";
    case AF2_ERR_NO_DEVICE: return "no usable device";
  }
  return "unknown status";
}

af2_status af2_create(int device_ordinal, af2_ctx **out) {
  if (!out) return AF2_ERR_INVALID_ARGUMENT;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    cudaGetLastError();
    return AF2_ERR_NO_DEVICE;
  }
  if (device_ordinal < 0 || device_ordinal >= count) return AF2_ERR_INVALID_ARGUMENT;
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device_ordinal) != cudaSuccess) return AF2_ERR_NO_DEVICE;
  if (prop.major != 10) return AF2_ERR_NO_DEVICE;  // built for sm_100a only
  if (cudaSetDevice(device_ordinal) != cudaSuccess) return AF2_ERR_NO_DEVICE;
  af2_ctx *ctx = new af2_ctx();
  ctx->device = device_ordinal;
  ctx->sm_count = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->err_word, sizeof(unsigned int)) != cudaSuccess ||
      cudaMemset(ctx->err_word, 0, sizeof(unsigned int)) != cudaSuccess ||
      cudaEventCreate(&ctx->ev_start) != cudaSuccess || cudaEventCreate(&ctx->ev_stop) != cudaSuccess) {
    af2_destroy(ctx);
    return AF2_ERR_CUDA;
  }
  *out = ctx;
  return AF2_OK;
}

void af2_destroy(af2_ctx *ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  comm_destroy(ctx);
  clear_weight_cache(ctx);
  if (ctx->workspace.ptr) cudaFree(ctx->workspace.ptr);
  for (auto &s : ctx->staging)
    if (s.ptr) cudaFree(s.ptr);
  if (ctx->err_word) cudaFree(ctx->err_word);
  for (const ProfilePending &p : ctx->pending) {
    cudaEventDestroy(p.start);
    cudaEventDestroy(p.stop);
  }
  for (cudaEvent_t e : ctx->free_events) cudaEventDestroy(e);
  if (ctx->ev_start) cudaEventDestroy(ctx->ev_start);
  if (ctx->ev_stop) cudaEventDestroy(ctx->ev_stop);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  delete ctx;
}

const char *af2_last_error(const af2_ctx *ctx) { return ctx ? ctx->last_error.c_str() : "no context"; }

uint64_t af2_launch_count(const af2_ctx *ctx) { return ctx ? ctx->launches : 0; }

af2_status af2_set_gemm_precision(af2_ctx *ctx, int precision) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (precision != AF2_GEMM_MATRIX && precision != AF2_GEMM_F32)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "precision must be AF2_GEMM_MATRIX or AF2_GEMM_F32");
  ctx->gemm_precision = precision;
  return AF2_OK;
}

int af2_get_gemm_precision(const af2_ctx *ctx) { return ctx ? ctx->gemm_precision : AF2_GEMM_MATRIX; }

af2_status af2_set_weight_cache(af2_ctx *ctx, int enable) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  ctx->weight_cache = enable != 0;
  if (!ctx->weight_cache) clear_weight_cache(ctx);
  return AF2_OK;
}

af2_status af2_clear_weight_cache(af2_ctx *ctx) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  clear_weight_cache(ctx);
  return AF2_OK;
}

af2_status af2_memory_snapshot(const af2_ctx *ctx, uint64_t *current_bytes, uint64_t *peak_bytes) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (current_bytes) *current_bytes = ctx->allocated;
  if (peak_bytes) *peak_bytes = ctx->peak;
  return AF2_OK;
}

af2_status af2_sync(af2_ctx *ctx, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  cudaSetDevice(ctx->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  if (af2_status st = comm_wait(ctx, s, "stream synchronize"); st != AF2_OK) return st;
  return check_device_errors(ctx);
}

af2_status af2_comm_set_timeout(af2_ctx *ctx, double seconds) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (!(seconds >= 0) || !std::isfinite(seconds))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "the timeout must be finite and non-negative");
  ctx->comm_timeout_s = seconds;
  return AF2_OK;
}

af2_status af2_profile_enable(af2_ctx *ctx, int enable) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  ctx->profiling = enable != 0;
  return AF2_OK;
}

static af2_status profile_fold(af2_ctx *ctx) {
  cudaSetDevice(ctx->device);
  for (const ProfilePending &p : ctx->pending) {
    cudaError_t e = cudaEventSynchronize(p.stop);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "profile event");
    float ms = 0.f;
    cudaEventElapsedTime(&ms, p.start, p.stop);
    ctx->prof_launches[p.id]++;
    ctx->prof_ms[p.id] += ms;
    ctx->free_events.push_back(p.start);
    ctx->free_events.push_back(p.stop);
  }
  ctx->pending.clear();
  return AF2_OK;
}

af2_status af2_profile_reset(af2_ctx *ctx) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = profile_fold(ctx);
  for (int i = 0; i < kProfCount; ++i) {
    ctx->prof_launches[i] = 0;
    ctx->prof_ms[i] = 0;
  }
  return st;
}

const char *af2_profile_kernel_name(int index) { return profile_name(index); }

af2_status af2_profile_read(af2_ctx *ctx, const char *kernel, uint64_t *launches, double *milliseconds) {
  if (!ctx || !kernel || !launches || !milliseconds) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = profile_fold(ctx);
  if (st != AF2_OK) return st;
  for (int i = 0; i < kProfCount; ++i) {
    if (std::strcmp(kernel, profile_name(i)) == 0) {
      *launches = ctx->prof_launches[i];
      *milliseconds = ctx->prof_ms[i];
      return AF2_OK;
    }
  }
  return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string("unknown kernel label ") + kernel);
}

int64_t af2_triangle_weight_count(int64_t c_z, int64_t c_hidden) {
  return 2 * c_z + 4 * (c_hidden * c_z + c_hidden) + 2 * c_hidden + (c_z * c_hidden + c_z) + (c_z * c_z + c_z);
}

af2_status af2_triangle_check(int direction, const af2_triangle_shape *shape, int64_t weight_count, double epsilon,
                              char *message, size_t capacity) {
  af2_ctx scratch;  // carries the message only; no device is touched
  const af2_status st = validate_triangle(&scratch, direction, shape, weight_count, epsilon);
  if (message && capacity > 0) {
    std::strncpy(message, scratch.last_error.c_str(), capacity - 1);
    message[capacity - 1] = '\0';
  }
  return st;
}

af2_status af2_triangle_workspace_bytes(const af2_triangle_shape *shape, const af2_triangle_options *options,
                                        uint64_t *bytes) {
  if (!shape || !bytes || !positive_safe(shape->length) || !positive_safe(shape->c_z) ||
      !positive_safe(shape->c_hidden))
    return AF2_ERR_INVALID_ARGUMENT;
  // The z re-layout is sized in, whatever z's dtype turns out to be.
  const TriangleLayout L = triangle_layout(shape->length, shape->c_z, shape->c_hidden,
                                           options ? options->block_rows : 0, AF2_F32);
  *bytes = L.total;
  return AF2_OK;
}

af2_status af2_triangle_multiplication(af2_ctx *ctx, int direction, const af2_triangle_shape *shape, const void *z,
                                       int z_dtype, const float *mask, const float *packed_weights,
                                       int64_t weight_count, double epsilon, const af2_triangle_options *options,
                                       void *out, int out_dtype, void *workspace, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = validate_triangle(ctx, direction, shape, weight_count, epsilon);
  if (st != AF2_OK) return st;
  if (!z || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(z_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  if (options && options->block_rows < 0)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "blockRows must be a positive safe integer");
  cudaSetDevice(ctx->device);
  const TriangleLayout L = triangle_layout(shape->length, shape->c_z, shape->c_hidden,
                                           options ? options->block_rows : 0, z_dtype);
  void *ws = workspace;
  if (!ws) {
    st = ensure(ctx, ctx->workspace, L.total, "triangle scratch");
    if (st != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return triangle_launch(ctx, direction, L, z, z_dtype, mask, packed_weights, epsilon,
                         options ? options->residual : 0, out, out_dtype, ws, s);
}

// One tensor each (the reference's TensorStore records): f32, or int8 codes with f16 block scales.
static af2_status validate_tensors(af2_ctx *ctx, const af2_matrix *tensors, int count, const char *op) {
  if (!tensors) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, std::string(op) + " weight tensors are NULL");
  for (int t = 0; t < count; ++t) {
    const af2_matrix &m = tensors[t];
    const std::string name = std::string(op) + " weight tensor " + std::to_string(t);
    if (m.format == AF2_WEIGHTS_Q8_CHANNEL)
      return fail(ctx, AF2_ERR_UNSUPPORTED, name + ": per-channel q8 is for the transition's matrices only");
    if (af2_status st = validate_matrix(ctx, m, name.c_str()); st != AF2_OK) return st;
    if (m.format == AF2_WEIGHTS_F32 && reinterpret_cast<uintptr_t>(m.values) % 4 != 0)
      return fail(ctx, AF2_ERR_INVALID_ARGUMENT, name + ": f32 values must be 4-byte aligned");
    if (m.format == AF2_WEIGHTS_Q8_BLOCK && reinterpret_cast<uintptr_t>(m.scales) % 2 != 0)
      return fail(ctx, AF2_ERR_INVALID_ARGUMENT, name + ": scales must be 2-byte aligned");
  }
  return AF2_OK;
}

af2_status af2_triangle_multiplication_weights(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                               const void *z, int z_dtype, const float *mask,
                                               const af2_matrix *tensors, double epsilon,
                                               const af2_triangle_options *options, void *out, int out_dtype,
                                               void *workspace, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = shape ? validate_triangle(ctx, direction, shape, af2_triangle_weight_count(shape->c_z, shape->c_hidden),
                                            epsilon)
                        : fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape is NULL");
  if (st != AF2_OK) return st;
  if ((st = validate_tensors(ctx, tensors, AF2_TRIANGLE_TENSORS, "triangle")) != AF2_OK) return st;
  if (!z || !mask || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(z_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  if (options && options->block_rows < 0)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "blockRows must be a positive safe integer");
  cudaSetDevice(ctx->device);
  const TriangleLayout L = triangle_layout(shape->length, shape->c_z, shape->c_hidden,
                                           options ? options->block_rows : 0, z_dtype);
  void *ws = workspace;
  if (!ws) {
    if ((st = ensure(ctx, ctx->workspace, L.total, "triangle scratch")) != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return triangle_launch(ctx, direction, L, z, z_dtype, mask, nullptr, epsilon, options ? options->residual : 0, out,
                         out_dtype, ws, s, nullptr, true, tensors);
}

af2_status af2_triangle_multiplication_host(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                            const void *z, const float *mask, const float *packed_weights,
                                            int64_t weight_count, double epsilon,
                                            const af2_triangle_options *options, int io_dtype, void *out,
                                            af2_op_stats *stats) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = validate_triangle(ctx, direction, shape, weight_count, epsilon);
  if (st != AF2_OK) return st;
  if (!z || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(io_dtype)) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  cudaSetDevice(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  const size_t pairs = (size_t)shape->length * shape->length;
  const size_t z_bytes = pairs * shape->c_z * dtype_bytes(io_dtype);
  const size_t mask_bytes = pairs * sizeof(float);
  const size_t w_bytes = (size_t)weight_count * sizeof(float);
  if ((st = ensure(ctx, ctx->staging[0], z_bytes, "z upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[1], mask_bytes, "mask upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[2], w_bytes, "weight upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[3], z_bytes, "output")) != AF2_OK)
    return st;
  const TriangleLayout L = triangle_layout(shape->length, shape->c_z, shape->c_hidden,
                                           options ? options->block_rows : 0, io_dtype);
  if ((st = ensure(ctx, ctx->workspace, L.total, "triangle scratch")) != AF2_OK) return st;
  cudaStream_t s = ctx->stream;
  const int residual = options ? options->residual : 0;
  cudaError_t e;
  if ((e = cudaMemcpyAsync(ctx->staging[0].ptr, z, z_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[1].ptr, mask, mask_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[2].ptr, packed_weights, w_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "upload inputs");
  if (residual &&
      (e = cudaMemcpyAsync(ctx->staging[3].ptr, ctx->staging[0].ptr, z_bytes, cudaMemcpyDeviceToDevice, s)) !=
          cudaSuccess)
    return cuda_fail(ctx, e, "seed residual output");
  cudaEventRecord(ctx->ev_start, s);
  st = triangle_launch(ctx, direction, L, ctx->staging[0].ptr, io_dtype, static_cast<const float *>(ctx->staging[1].ptr),
                       static_cast<const float *>(ctx->staging[2].ptr), epsilon, residual, ctx->staging[3].ptr,
                       io_dtype, ctx->workspace.ptr, s);
  if (st != AF2_OK) return st;
  cudaEventRecord(ctx->ev_stop, s);
  if ((e = cudaMemcpyAsync(out, ctx->staging[3].ptr, z_bytes, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "read back output");
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(ctx, e, "triangle multiplication");
  if ((st = check_device_errors(ctx)) != AF2_OK) return st;
  if (stats) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop);
    const double n = (double)shape->length, cz = (double)shape->c_z, ch = (double)shape->c_hidden;
    stats->device_milliseconds = ms;
    stats->host_milliseconds =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    // kernel-cost.ts:158-162: gate, block + whole projections, contraction, output.
    stats->flops = 2 * n * n * (cz * cz + 2 * cz * 2 * ch + n * ch + ch * cz);
    stats->workspace_bytes = L.total;
    stats->peak_bytes = ctx->peak;
  }
  return AF2_OK;
}

int64_t af2_transition_weight_count(int64_t channels, int64_t hidden_channels) {
  return 2 * channels + channels * hidden_channels + hidden_channels + hidden_channels * channels + channels;
}

af2_status af2_transition_check(const af2_transition_shape *shape, int64_t weight_count, double epsilon,
                                char *message, size_t capacity) {
  af2_ctx scratch;
  af2_status st = validate_transition(&scratch, shape, epsilon);
  if (st == AF2_OK) {
    const int64_t expected = af2_transition_weight_count(shape->channels, shape->hidden_channels);
    if (weight_count != expected)
      st = fail(&scratch, AF2_ERR_INVALID_ARGUMENT, "packed weights have " + std::to_string(weight_count) +
                                                        " values; expected " + std::to_string(expected));
  }
  if (message && capacity > 0) {
    std::strncpy(message, scratch.last_error.c_str(), capacity - 1);
    message[capacity - 1] = '\0';
  }
  return st;
}

af2_status af2_transition_workspace_bytes(const af2_transition_shape *shape, uint64_t *bytes) {
  if (!shape || !bytes || !positive_safe(shape->rows) || !positive_safe(shape->channels) ||
      !positive_safe(shape->hidden_channels))
    return AF2_ERR_INVALID_ARGUMENT;
  // Sized for the normalised copy too, whatever x's dtype turns out to be.
  *bytes = transition_layout(shape->rows, shape->channels, shape->hidden_channels, AF2_F32).total;
  return AF2_OK;
}

af2_status af2_transition(af2_ctx *ctx, const af2_transition_shape *shape, const void *x, int x_dtype,
                          const af2_transition_weights *weights, double epsilon, const af2_transition_options *options,
                          void *out, int out_dtype, void *workspace, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = validate_transition(ctx, shape, epsilon);
  if (st != AF2_OK) return st;
  if (!x || !out || !weights) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!weights->layer_norm_scale || !weights->layer_norm_offset || !weights->first_bias || !weights->second_bias)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a weight vector is NULL");
  if ((st = validate_matrix(ctx, weights->first_weight, "firstWeight")) != AF2_OK ||
      (st = validate_matrix(ctx, weights->second_weight, "secondWeight")) != AF2_OK)
    return st;
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  if (options && options->max_chunk_rows < 0)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "maxChunkRows must be a positive safe integer");
  cudaSetDevice(ctx->device);
  const TransitionLayout L = transition_layout(shape->rows, shape->channels, shape->hidden_channels, x_dtype);
  void *ws = workspace;
  if (!ws) {
    if ((st = ensure(ctx, ctx->workspace, L.total, "transition scratch")) != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return transition_launch(ctx, L, x, x_dtype, *weights, epsilon, options ? options->residual : 0, out, out_dtype,
                           ws, s);
}

af2_status af2_transition_host(af2_ctx *ctx, const af2_transition_shape *shape, const void *x,
                               const float *packed_weights, int64_t weight_count, double epsilon,
                               const af2_transition_options *options, int io_dtype, void *out, af2_op_stats *stats) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = validate_transition(ctx, shape, epsilon);
  if (st != AF2_OK) return st;
  const int64_t expected = af2_transition_weight_count(shape->channels, shape->hidden_channels);
  if (weight_count != expected)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "packed weights have " + std::to_string(weight_count) +
                                                   " values; expected " + std::to_string(expected));
  if (!x || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(io_dtype)) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  if (options && options->max_chunk_rows < 0)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "maxChunkRows must be a positive safe integer");
  cudaSetDevice(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  const int64_t c = shape->channels, h = shape->hidden_channels;
  const size_t x_bytes = (size_t)shape->rows * c * dtype_bytes(io_dtype);
  const size_t w_bytes = (size_t)weight_count * sizeof(float);
  if ((st = ensure(ctx, ctx->staging[0], x_bytes, "x upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[2], w_bytes, "weight upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[3], x_bytes, "output")) != AF2_OK)
    return st;
  const TransitionLayout L = transition_layout(shape->rows, c, h, io_dtype);
  if ((st = ensure(ctx, ctx->workspace, L.total, "transition scratch")) != AF2_OK) return st;
  cudaStream_t s = ctx->stream;
  const int residual = options ? options->residual : 0;
  cudaError_t e;
  if ((e = cudaMemcpyAsync(ctx->staging[0].ptr, x, x_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[2].ptr, packed_weights, w_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "upload inputs");
  if (residual &&
      (e = cudaMemcpyAsync(ctx->staging[3].ptr, ctx->staging[0].ptr, x_bytes, cudaMemcpyDeviceToDevice, s)) !=
          cudaSuccess)
    return cuda_fail(ctx, e, "seed residual output");
  // packTransitionWeights order (transition.ts:140-177): LN scale, LN offset, W1, b1, W2, b2.
  const float *pw = static_cast<const float *>(ctx->staging[2].ptr);
  af2_transition_weights w{};
  w.layer_norm_scale = pw;
  w.layer_norm_offset = pw + c;
  w.first_weight = af2_matrix{AF2_WEIGHTS_F32, 0, pw + 2 * c, nullptr};
  w.first_bias = pw + 2 * c + c * h;
  w.second_weight = af2_matrix{AF2_WEIGHTS_F32, 0, pw + 2 * c + c * h + h, nullptr};
  w.second_bias = pw + 2 * c + 2 * c * h + h;
  cudaEventRecord(ctx->ev_start, s);
  st = transition_launch(ctx, L, ctx->staging[0].ptr, io_dtype, w, epsilon, residual, ctx->staging[3].ptr, io_dtype,
                         ctx->workspace.ptr, s);
  if (st != AF2_OK) return st;
  cudaEventRecord(ctx->ev_stop, s);
  if ((e = cudaMemcpyAsync(out, ctx->staging[3].ptr, x_bytes, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "read back output");
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(ctx, e, "transition");
  if ((st = check_device_errors(ctx)) != AF2_OK) return st;
  if (stats) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop);
    stats->device_milliseconds = ms;
    stats->host_milliseconds =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    // kernel-cost.ts: two GEMMs, rows x C x H each.
    stats->flops = 4.0 * (double)shape->rows * (double)c * (double)h;
    stats->workspace_bytes = L.total;
    stats->peak_bytes = ctx->peak;
  }
  return AF2_OK;
}

af2_status af2_dequant_q8(af2_ctx *ctx, const af2_matrix *matrix, int64_t inner, int64_t cols, float *out,
                          void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (!matrix || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "matrix or output is NULL");
  if (!positive_safe(inner) || !positive_safe(cols))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "matrix dimensions must be positive safe integers");
  if (matrix->format != AF2_WEIGHTS_Q8_BLOCK && matrix->format != AF2_WEIGHTS_Q8_CHANNEL)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "af2_dequant_q8 decodes q8 matrices only");
  af2_status st = validate_matrix(ctx, *matrix, "matrix");
  if (st != AF2_OK) return st;
  cudaSetDevice(ctx->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return dequant_launch(ctx, *matrix, inner, cols, out, s);
}

int64_t af2_opm_weight_count(const af2_opm_shape *shape) {
  if (!shape) return 0;
  const int64_t cm = shape->c_m, c = shape->c_outer, cz = shape->c_z;
  return 2 * cm + 2 * (cm * c + c) + c * c * cz + cz;
}

af2_status af2_opm_check(const af2_opm_shape *shape, int64_t weight_count, char *message, size_t capacity) {
  af2_ctx scratch;
  const af2_status st = validate_opm(&scratch, shape, weight_count);
  if (message && capacity > 0) {
    std::strncpy(message, scratch.last_error.c_str(), capacity - 1);
    message[capacity - 1] = '\0';
  }
  return st;
}

af2_status af2_opm_workspace_bytes(const af2_opm_shape *shape, const af2_opm_options *options, uint64_t *bytes) {
  if (!shape || !bytes) return AF2_ERR_INVALID_ARGUMENT;
  af2_ctx scratch;
  if (validate_opm(&scratch, shape, af2_opm_weight_count(shape)) != AF2_OK) return AF2_ERR_INVALID_ARGUMENT;
  // for the default GEMM precision (the f32 mode takes context-owned scratch only)
  *bytes = opm_layout(shape->sequences, shape->length, shape->c_m, shape->c_outer, shape->c_z,
                      options ? options->row_block_residues : 0)
               .total;
  return AF2_OK;
}

static af2_status opm_options(af2_ctx *ctx, const af2_opm_options *o, double *ln_eps, double *norm_eps, int *rb,
                              int *residual) {
  *ln_eps = (o && o->layer_norm_epsilon != 0) ? o->layer_norm_epsilon : 1e-5;
  *norm_eps = (o && o->normalization_epsilon != 0) ? o->normalization_epsilon : 1e-3;
  *rb = o ? o->row_block_residues : 0;
  *residual = o ? o->residual : 0;
  if (!(*ln_eps > 0) || !std::isfinite(*ln_eps) || !(*norm_eps > 0) || !std::isfinite(*norm_eps))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "epsilons must be finite and positive");
  if (*rb < 0) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "rowBlockResidues must be a positive safe integer");
  return AF2_OK;
}

af2_status af2_outer_product_mean(af2_ctx *ctx, const af2_opm_shape *shape, const void *m, int m_dtype,
                                  const float *mask, const float *packed_weights, int64_t weight_count,
                                  const af2_opm_options *options, void *out, int out_dtype, void *workspace,
                                  void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = validate_opm(ctx, shape, weight_count);
  if (st != AF2_OK) return st;
  if (!m || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(m_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  double ln_eps, norm_eps;
  int rb, residual;
  if ((st = opm_options(ctx, options, &ln_eps, &norm_eps, &rb, &residual)) != AF2_OK) return st;
  cudaSetDevice(ctx->device);
  const OpmLayout L = opm_layout(shape->sequences, shape->length, shape->c_m, shape->c_outer, shape->c_z, rb, 0, 0,
                                 ctx->gemm_precision == AF2_GEMM_F32);
  void *ws = workspace;
  if (ws && L.split)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT,
                "in the AF2_GEMM_F32 precision the outer product mean takes context-owned scratch (workspace NULL)");
  if (!ws) {
    if ((st = ensure(ctx, ctx->workspace, L.total, "outer product mean scratch")) != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return opm_launch(ctx, L, m, m_dtype, mask, packed_weights, ln_eps, norm_eps, residual, out, out_dtype, ws, s);
}

af2_status af2_outer_product_mean_weights(af2_ctx *ctx, const af2_opm_shape *shape, const void *m, int m_dtype,
                                          const float *mask, const af2_matrix *tensors,
                                          const af2_opm_options *options, void *out, int out_dtype, void *workspace,
                                          void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (!shape) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape is NULL");
  af2_status st = validate_opm(ctx, shape, af2_opm_weight_count(shape));
  if (st != AF2_OK) return st;
  if ((st = validate_tensors(ctx, tensors, AF2_OPM_TENSORS, "outer product mean")) != AF2_OK) return st;
  if (!m || !mask || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(m_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  double ln_eps, norm_eps;
  int rb, residual;
  if ((st = opm_options(ctx, options, &ln_eps, &norm_eps, &rb, &residual)) != AF2_OK) return st;
  cudaSetDevice(ctx->device);
  const OpmLayout L = opm_layout(shape->sequences, shape->length, shape->c_m, shape->c_outer, shape->c_z, rb, 0, 0,
                                 ctx->gemm_precision == AF2_GEMM_F32);
  void *ws = workspace;
  if (ws && L.split)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT,
                "in the AF2_GEMM_F32 precision the outer product mean takes context-owned scratch (workspace NULL)");
  if (!ws) {
    if ((st = ensure(ctx, ctx->workspace, L.total, "outer product mean scratch")) != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return opm_launch(ctx, L, m, m_dtype, mask, nullptr, ln_eps, norm_eps, residual, out, out_dtype, ws, s, nullptr,
                    tensors);
}

af2_status af2_outer_product_mean_host(af2_ctx *ctx, const af2_opm_shape *shape, const void *m, const float *mask,
                                       const float *packed_weights, int64_t weight_count,
                                       const af2_opm_options *options, int io_dtype, void *out, af2_op_stats *stats) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  af2_status st = validate_opm(ctx, shape, weight_count);
  if (st != AF2_OK) return st;
  if (!m || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(io_dtype)) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  double ln_eps, norm_eps;
  int rb, residual;
  if ((st = opm_options(ctx, options, &ln_eps, &norm_eps, &rb, &residual)) != AF2_OK) return st;
  cudaSetDevice(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  const int64_t S = shape->sequences, N = shape->length;
  const size_t m_bytes = (size_t)S * N * shape->c_m * dtype_bytes(io_dtype);
  const size_t mask_bytes = (size_t)S * N * sizeof(float);
  const size_t w_bytes = (size_t)weight_count * sizeof(float);
  const size_t out_bytes = (size_t)N * N * shape->c_z * dtype_bytes(io_dtype);
  if ((st = ensure(ctx, ctx->staging[0], m_bytes, "m upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[1], mask_bytes, "mask upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[2], w_bytes, "weight upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[3], out_bytes, "output")) != AF2_OK)
    return st;
  const OpmLayout L = opm_layout(S, N, shape->c_m, shape->c_outer, shape->c_z, rb, 0, 0,
                                 ctx->gemm_precision == AF2_GEMM_F32);
  if ((st = ensure(ctx, ctx->workspace, L.total, "outer product mean scratch")) != AF2_OK) return st;
  cudaStream_t s = ctx->stream;
  cudaError_t e;
  if ((e = cudaMemcpyAsync(ctx->staging[0].ptr, m, m_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[1].ptr, mask, mask_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[2].ptr, packed_weights, w_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "upload inputs");
  if (residual && (e = cudaMemsetAsync(ctx->staging[3].ptr, 0, out_bytes, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "clear residual output");
  cudaEventRecord(ctx->ev_start, s);
  st = opm_launch(ctx, L, ctx->staging[0].ptr, io_dtype, static_cast<const float *>(ctx->staging[1].ptr),
                  static_cast<const float *>(ctx->staging[2].ptr), ln_eps, norm_eps, residual, ctx->staging[3].ptr,
                  io_dtype, ctx->workspace.ptr, s);
  if (st != AF2_OK) return st;
  cudaEventRecord(ctx->ev_stop, s);
  if ((e = cudaMemcpyAsync(out, ctx->staging[3].ptr, out_bytes, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "read back output");
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(ctx, e, "outer product mean");
  if ((st = check_device_errors(ctx)) != AF2_OK) return st;
  if (stats) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop);
    const double dS = (double)S, dN = (double)N, cm = (double)shape->c_m, c = (double)shape->c_outer,
                 cz = (double)shape->c_z;
    stats->device_milliseconds = ms;
    stats->host_milliseconds =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    // kernel-cost.ts: projection 2 S N c_m 2c, contraction 2 (N c)^2 S, output 2 N^2 c^2 c_z.
    stats->flops = 2 * dS * dN * cm * 2 * c + 2 * dN * c * dN * c * dS + 2 * dN * dN * c * c * cz;
    stats->workspace_bytes = L.total;
    stats->peak_bytes = ctx->peak;
  }
  return AF2_OK;
}

int64_t af2_attention_weight_count(const af2_attention_shape *shape, int pair_bias) {
  if (!shape) return 0;
  const int64_t c = shape->channels;
  return 2 * c + 4 * c * c + c + c * c + c + (pair_bias == AF2_PAIR_BIAS_NORMALIZED_INPUT ? c * shape->heads : 0);
}

}  // extern "C"

namespace af2 {
namespace {
// validate (src/evoformer/attention.ts:102-141) for a C caller, then the kernels' limits.
af2_status validate_attention(af2_ctx *ctx, const af2_attention_shape *shape, int pair_bias, int64_t weight_count,
                              double epsilon) {
  if (!shape) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape is NULL");
  if (!positive_safe(shape->batch) || !positive_safe(shape->queries) || !positive_safe(shape->channels) ||
      !positive_safe(shape->heads))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "attention dimensions must be positive safe integers");
  if (shape->channels % shape->heads != 0 || shape->channels / shape->heads > 32)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT,
                "the fused WebGPU attention path requires an integral head dimension no larger than 32");
  if (pair_bias != AF2_PAIR_BIAS_NONE && pair_bias != AF2_PAIR_BIAS_NORMALIZED_INPUT)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "pair_bias must be AF2_PAIR_BIAS_NONE or AF2_PAIR_BIAS_NORMALIZED_INPUT");
  if ((double)shape->batch * (double)shape->queries * (double)shape->channels > (double)kMaxSafeInteger)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "tensor dimensions exceed JavaScript's safe integer range");
  const int64_t expected = af2_attention_weight_count(shape, pair_bias);
  if (weight_count != expected)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "packed weights have " + std::to_string(weight_count) +
                                                   " values; expected " + std::to_string(expected));
  if (!(epsilon > 0) || !std::isfinite(epsilon))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "epsilon must be finite and positive; received " +
                                                   std::to_string(epsilon));
  if (shape->channels / shape->heads != 32)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "the sm_100a attention kernel is built for a head dimension of 32");
  if (shape->channels > 256) return fail(ctx, AF2_ERR_UNSUPPORTED, "attention channels above 256 are not supported");
  if (pair_bias == AF2_PAIR_BIAS_NORMALIZED_INPUT && shape->batch != shape->queries)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "a normalized-input pair bias needs batch == queries (triangle attention)");
  if (shape->queries > (int64_t(1) << 20) || shape->batch > (int64_t(1) << 20) ||
      shape->batch * shape->queries > (int64_t(1) << 31))
    return fail(ctx, AF2_ERR_UNSUPPORTED, "attention beyond 2^31 rows is not supported");
  return AF2_OK;
}
}  // namespace
}  // namespace af2

extern "C" {

af2_status af2_attention_check(const af2_attention_shape *shape, int pair_bias, int64_t weight_count, double epsilon,
                               char *message, size_t capacity) {
  af2_ctx scratch;
  const af2_status st = validate_attention(&scratch, shape, pair_bias, weight_count, epsilon);
  if (message && capacity > 0) {
    std::strncpy(message, scratch.last_error.c_str(), capacity - 1);
    message[capacity - 1] = '\0';
  }
  return st;
}

af2_status af2_attention_workspace_bytes(const af2_attention_shape *shape, int pair_bias, uint64_t *bytes) {
  if (!shape || !bytes) return AF2_ERR_INVALID_ARGUMENT;
  af2_ctx scratch;
  if (validate_attention(&scratch, shape, pair_bias, af2_attention_weight_count(shape, pair_bias), 1e-5) != AF2_OK)
    return AF2_ERR_INVALID_ARGUMENT;
  *bytes = attention_layout(shape->batch, shape->queries, shape->channels, shape->heads,
                            pair_bias == AF2_PAIR_BIAS_NORMALIZED_INPUT)
               .total;
  return AF2_OK;
}

af2_status af2_attention(af2_ctx *ctx, const af2_attention_shape *shape, const void *x, int x_dtype, const float *mask,
                         const float *packed_weights, int64_t weight_count, double epsilon,
                         const af2_attention_options *options, void *out, int out_dtype, void *workspace,
                         void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  const int pair_bias = options ? options->pair_bias : AF2_PAIR_BIAS_NONE;
  af2_status st = validate_attention(ctx, shape, pair_bias, weight_count, epsilon);
  if (st != AF2_OK) return st;
  if (!x || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  if (!valid_dtype(x_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  cudaSetDevice(ctx->device);
  const AttentionLayout L = attention_layout(shape->batch, shape->queries, shape->channels, shape->heads,
                                             pair_bias == AF2_PAIR_BIAS_NORMALIZED_INPUT);
  void *ws = workspace;
  if (!ws) {
    if ((st = ensure(ctx, ctx->workspace, L.total, "attention scratch")) != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return attention_launch(ctx, L, options ? options->transpose : 0, x, x_dtype, mask, packed_weights, epsilon,
                          options ? options->residual : 0, out, out_dtype, ws, s);
}

af2_status af2_attention_host(af2_ctx *ctx, const af2_attention_shape *shape, const float *x, const float *mask,
                              const float *packed_weights, int64_t weight_count, double epsilon,
                              const af2_attention_options *options, float *out, af2_op_stats *stats) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  const int pair_bias = options ? options->pair_bias : AF2_PAIR_BIAS_NONE;
  af2_status st = validate_attention(ctx, shape, pair_bias, weight_count, epsilon);
  if (st != AF2_OK) return st;
  if (!x || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  cudaSetDevice(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  const size_t rows = (size_t)shape->batch * shape->queries;
  const size_t x_bytes = rows * shape->channels * sizeof(float), mask_bytes = rows * sizeof(float),
               w_bytes = (size_t)weight_count * sizeof(float);
  if ((st = ensure(ctx, ctx->staging[0], x_bytes, "x upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[1], mask_bytes, "mask upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[2], w_bytes, "weight upload")) != AF2_OK ||
      (st = ensure(ctx, ctx->staging[3], x_bytes, "output")) != AF2_OK)
    return st;
  const AttentionLayout L = attention_layout(shape->batch, shape->queries, shape->channels, shape->heads,
                                             pair_bias == AF2_PAIR_BIAS_NORMALIZED_INPUT);
  if ((st = ensure(ctx, ctx->workspace, L.total, "attention scratch")) != AF2_OK) return st;
  cudaStream_t s = ctx->stream;
  const int residual = options ? options->residual : 0;
  cudaError_t e;
  if ((e = cudaMemcpyAsync(ctx->staging[0].ptr, x, x_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[1].ptr, mask, mask_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess ||
      (e = cudaMemcpyAsync(ctx->staging[2].ptr, packed_weights, w_bytes, cudaMemcpyHostToDevice, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "upload inputs");
  if (residual &&
      (e = cudaMemcpyAsync(ctx->staging[3].ptr, ctx->staging[0].ptr, x_bytes, cudaMemcpyDeviceToDevice, s)) !=
          cudaSuccess)
    return cuda_fail(ctx, e, "seed residual output");
  cudaEventRecord(ctx->ev_start, s);
  st = attention_launch(ctx, L, options ? options->transpose : 0, ctx->staging[0].ptr, AF2_F32,
                        static_cast<const float *>(ctx->staging[1].ptr), static_cast<const float *>(ctx->staging[2].ptr),
                        epsilon, residual, ctx->staging[3].ptr, AF2_F32, ctx->workspace.ptr, s);
  if (st != AF2_OK) return st;
  cudaEventRecord(ctx->ev_stop, s);
  if ((e = cudaMemcpyAsync(out, ctx->staging[3].ptr, x_bytes, cudaMemcpyDeviceToHost, s)) != cudaSuccess)
    return cuda_fail(ctx, e, "read back output");
  if ((e = cudaStreamSynchronize(s)) != cudaSuccess) return cuda_fail(ctx, e, "attention");
  if ((st = check_device_errors(ctx)) != AF2_OK) return st;
  if (stats) {
    float ms = 0.f;
    cudaEventElapsedTime(&ms, ctx->ev_start, ctx->ev_stop);
    const double r = (double)rows, c = (double)shape->channels, h = (double)shape->heads,
                 q = (double)shape->queries;
    stats->device_milliseconds = ms;
    stats->host_milliseconds =
        std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
    // kernel-cost.ts:79-92: project gemm(rows, C, 4C), flash 2 gemm(rows H, 32, Q), output gemm(rows, C, C),
    // pair bias gemm(rows, C, H)
    stats->flops = 2 * r * c * 4 * c + 4 * r * h * 32 * q + 2 * r * c * c +
                   (pair_bias == AF2_PAIR_BIAS_NORMALIZED_INPUT ? 2 * r * c * h : 0);
    stats->workspace_bytes = L.total;
    stats->peak_bytes = ctx->peak;
  }
  return AF2_OK;
}

af2_status af2_linear_workspace_bytes(const af2_linear_shape *shape, int a_dtype, uint64_t *bytes) {
  if (!shape || !bytes || !positive_safe(shape->rows) || !positive_safe(shape->inner) ||
      !positive_safe(shape->columns))
    return AF2_ERR_INVALID_ARGUMENT;
  *bytes = linear_layout(shape->rows, shape->inner, shape->columns, a_dtype).total;
  return AF2_OK;
}

af2_status af2_linear(af2_ctx *ctx, const af2_linear_shape *shape, const void *a, int a_dtype,
                      const af2_matrix *weight, const float *bias, int activation, int residual, void *out,
                      int out_dtype, void *workspace, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (!shape || !positive_safe(shape->rows) || !positive_safe(shape->inner) || !positive_safe(shape->columns))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "linear dimensions must be positive safe integers");
  if (!a || !weight || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  af2_status st = validate_matrix(ctx, *weight, "weight");
  if (st != AF2_OK) return st;
  if (!valid_dtype(a_dtype) || !valid_dtype(out_dtype))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  if (activation != AF2_ACTIVATION_NONE && activation != AF2_ACTIVATION_RELU)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "activation must be AF2_ACTIVATION_NONE or AF2_ACTIVATION_RELU");
  if (shape->rows > (int64_t(1) << 31) - 256 || shape->inner > 65536 || shape->columns > 65536)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "linear layer beyond 2^31 rows or 65536 channels");
  cudaSetDevice(ctx->device);
  const LinearLayout L = linear_layout(shape->rows, shape->inner, shape->columns, a_dtype);
  void *ws = workspace;
  if (!ws) {
    if ((st = ensure(ctx, ctx->workspace, L.total, "linear scratch")) != AF2_OK) return st;
    ws = ctx->workspace.ptr;
  } else if (reinterpret_cast<uintptr_t>(ws) % 256 != 0) {
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "workspace must be 256-byte aligned");
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return linear_run(ctx, L, shape->rows, shape->inner, shape->columns, a, a_dtype, *weight, bias, activation,
                    residual, out, out_dtype, ws, s);
}

}  // extern "C"
