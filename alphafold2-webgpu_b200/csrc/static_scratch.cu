// static_scratch.cu -- triangle multiplication whose scratch lives in a fixed
// device array instead of memory the library allocates.
//
// Some hosts cannot let a library call cudaMalloc: a host whose own memory
// manager owns the device under a fixed budget (the reference's allocator
// rejects anything over its budget, src/runtime/allocator.ts:76-90), and
// latency-sensitive callers for which cudaMalloc and cudaFree are ruled out
// because they can synchronise the device and stall other streams.
// af2_triangle_multiplication_static gives them the device-form triangle
// update with its scratch (prepared weights, the projected operands and the
// contracted block) taken from kScratchBytes of file-scope device memory.
//
// That array exists on every GPU where the library's module is loaded and is
// held until the process exits.  Every call shares it, so calls whose work
// overlaps on the GPU (two streams, or two host threads) race on it.  Nothing
// in it has to start at zero: each byte a kernel reads is written earlier in
// the same call, so the contents a previous call left behind do not matter.
#include <mutex>
#include <string>

#include "af2_internal.h"

namespace af2 {
namespace {

// 16.5 MiB: the whole scratch of one call at length <= 128 with
// c_z = c_hidden = 128 (f32 z included, which needs an f16 copy).
constexpr size_t kScratchBytes = 16896u * 1024u;
static __device__ __align__(256) unsigned char g_triangle_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
void *g_scratch_address[kMaxDevices] = {};

// The array's name is only a host-side stand-in: the kernels need its device
// address, looked up once per device with that device current.  The address is
// kept for the life of the process, so a cudaDeviceReset while the library is
// loaded is not supported: the kept address would belong to the destroyed context.
af2_status scratch_address(af2_ctx *ctx, void **out) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices)
    return fail(ctx, AF2_ERR_UNSUPPORTED, "device ordinal beyond the static scratch table");
  std::lock_guard<std::mutex> lock(g_setup_mutex);
  if (!g_scratch_address[ctx->device]) {
    void *ptr = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&ptr, g_triangle_scratch);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "look up the static triangle scratch");
    g_scratch_address[ctx->device] = ptr;
  }
  *out = g_scratch_address[ctx->device];
  return AF2_OK;
}

}  // namespace
}  // namespace af2

using namespace af2;

extern "C" af2_status af2_triangle_multiplication_static(af2_ctx *ctx, int direction, const af2_triangle_shape *shape,
                                                         const void *z, int z_dtype, const float *mask,
                                                         const float *packed_weights, int64_t weight_count,
                                                         double epsilon, const af2_triangle_options *options,
                                                         void *out, int out_dtype, void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  char message[256];
  af2_status st = af2_triangle_check(direction, shape, weight_count, epsilon, message, sizeof message);
  if (st != AF2_OK) return fail(ctx, st, message);
  if (!z || !mask || !packed_weights || !out) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a tensor pointer is NULL");
  const bool dtypes_ok = (z_dtype == AF2_F32 || z_dtype == AF2_F16 || z_dtype == AF2_BF16) &&
                         (out_dtype == AF2_F32 || out_dtype == AF2_F16 || out_dtype == AF2_BF16);
  if (!dtypes_ok) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  if (options && options->block_rows < 0)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "blockRows must be a positive safe integer");
  const TriangleLayout L = triangle_layout(shape->length, shape->c_z, shape->c_hidden,
                                           options ? options->block_rows : 0, z_dtype);
  if (L.total > kScratchBytes)
    return fail(ctx, AF2_ERR_UNSUPPORTED,
                "this shape needs " + std::to_string(L.total) + " bytes of scratch; the static scratch holds " +
                    std::to_string(kScratchBytes) + " bytes (length <= 128 at c_z = c_hidden = 128); use "
                    "af2_triangle_multiplication for larger shapes");
  cudaError_t e = cudaSetDevice(ctx->device);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "select the context's device");
  void *scratch = nullptr;
  if ((st = scratch_address(ctx, &scratch)) != AF2_OK) return st;
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  return triangle_launch(ctx, direction, L, z, z_dtype, mask, packed_weights, epsilon,
                         options ? options->residual : 0, out, out_dtype, scratch, s, nullptr,
                         /*cache_weights=*/false);
}
