// triangle.cu -- triangle multiplication (outgoing and incoming) on sm_100a.
//
// Reference: src/triangle/cpu-reference.ts:56-100 (the maths),
// src/triangle/shaders.ts:151-589 (the seven WGSL kernels this replaces) and
// src/evoformer/block.ts:1497-1671 (the in-model encoder).
//
// Three persistent, warp-specialised kernels per call:
//
//  1. project  -- LayerNorm(z) on load, then the four c_z -> c_h projections
//     (a_p, a_g, b_p, b_g) as one tcgen05 GEMM per 64-pair tile, computed
//     transposed (D[h][pair] = W[h][:] . zn[pair][:]) so that a TMEM lane is a
//     hidden channel and the gated result a = mask (p + b_p) sigmoid(g + b_g)
//     is stored row-major [row][h][k] with 16-byte vector stores, so the rows
//     one rank of a row-sharded pair projects form one contiguous block.  The
//     incoming direction reads z in transposed pair order, so its operands
//     come out as a'[j][h][k] = a[k][j] and the contraction below is the same
//     NT GEMM for both directions.
//  2. contract -- per hidden channel h, X[h] = (1/N) A[h] B[h]^T with TMA-fed
//     256x256x64 tiles on CTA pairs, a 6-deep mbarrier pipeline and two TMEM accumulators
//     so the epilogue of one tile overlaps the MMAs of the next.  X is stored
//     f16, pre-scaled by 1/N so any N stays inside the f16 range.
//  3. output   -- per 128-pair tile: the [h][pair] block of X feeds the first
//     GEMM as it lands (MN-major), while four warps take its per-pair
//     LayerNorm statistics (eps scaled by 1/N^2 to undo the pre-scale); z is
//     layer-normalised again in place; two tcgen05 GEMMs give X W_z'^T and
//     LN(z) W_g^T, and the epilogue forms LN_out(X) W_z'^T =
//     rstd (X W_z'^T - mean rowsum(W_z')), applies the biases, the sigmoid
//     gate and the optional residual add and writes the pair rows.
//
// All channel dimensions are padded to 128 (weights zero-padded), with the
// LayerNorm statistics taken over the real channel counts.
#include "af2_device.cuh"
#include "af2_internal.h"

#include <algorithm>
#include <array>
#include <cstring>

namespace af2 {
namespace tri {

constexpr int C = 128;  // padded channel count of every triangle tile
constexpr int64_t kChannelPad = 64;  // elements added to every channel pitch

// Prepared weights: six [128][128] f16 matrices, [out][in] row-major.
enum { kWAP = 0, kWAG = 1, kWBP = 2, kWBG = 3, kWZ = 4, kWG = 5, kMatCount = 6 };
// Prepared vectors: 128 f32 each.
// kVZSum: per output channel, the sum over hidden channels of the f16-rounded
// W_z diag(gamma_out) row (the output kernel normalises X after its GEMM).
enum {
  kVLnInW = 0, kVLnInB, kVBAP, kVBAG, kVBBP, kVBBG, kVLnOutW, kVLnOutB, kVBZ, kVBG, kVZSum, kVecCount
};

// ---------------------------------------------------------------------------
// Weight preparation: the 16 tensors of the reference's ORDER
// (src/triangle/weights.ts:4-10) -> zero-padded f16 matrices + f32 vectors.
// They arrive either as the packed f32 array or as one tensor each, f32 or
// mixed-q8 (int8 codes with an f16 scale per 64-element block of the
// flattened tensor, src/reference/dtype.ts:86-97); q8 codes are decoded here,
// on the way into the f16 operands.
// ---------------------------------------------------------------------------
enum {
  kTLnInW = 0, kTLnInB, kTApW, kTApB, kTAgW, kTAgB, kTBpW, kTBpB, kTBgW, kTBgB, kTLnOutW, kTLnOutB, kTZW, kTZB,
  kTGW, kTGB, kTensorCount
};

// The packed f32 array: tensor t starts at offset[t].
struct PackedAccess {
  const float *packed;
  int64_t offset[kTensorCount];
  __device__ __forceinline__ float operator()(int t, int64_t i) const { return packed[offset[t] + i]; }
};

// One tensor each: f32 values or block-scaled int8 codes.
struct TensorAccess {
  const void *values[kTensorCount];
  const uint16_t *scales[kTensorCount];  // NULL: f32
  int block[kTensorCount];
  __device__ __forceinline__ float operator()(int t, int64_t i) const {
    if (!scales[t]) return static_cast<const float *>(values[t])[i];
    const float code = static_cast<float>(static_cast<const int8_t *>(values[t])[i]);
    return code * __half2float(__ushort_as_half(scales[t][i / block[t]]));
  }
};

template <typename Acc>
__global__ void prep_weights_kernel(const Acc w, int cz, int ch, __half *__restrict__ w16, float *__restrict__ vec) {
  // The LayerNorm affine maps are folded into the projections that follow
  // them: LN(x) W^T + b = ((x - mean) rstd) (W diag(gamma))^T + (b + W beta),
  // so the kernels normalise without gamma/beta and the weights carry them.
  const int stride = gridDim.x * blockDim.x;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < kMatCount * C * C; idx += stride) {
    const int m = idx / (C * C), r = (idx / C) % C, c = idx % C;
    float v = 0.f;
    switch (m) {
      case kWAP: if (r < ch && c < cz) v = w(kTApW, (int64_t)r * cz + c) * w(kTLnInW, c); break;
      case kWAG: if (r < ch && c < cz) v = w(kTAgW, (int64_t)r * cz + c) * w(kTLnInW, c); break;
      case kWBP: if (r < ch && c < cz) v = w(kTBpW, (int64_t)r * cz + c) * w(kTLnInW, c); break;
      case kWBG: if (r < ch && c < cz) v = w(kTBgW, (int64_t)r * cz + c) * w(kTLnInW, c); break;
      case kWZ: if (r < cz && c < ch) v = w(kTZW, (int64_t)r * ch + c) * w(kTLnOutW, c); break;
      default: if (r < cz && c < cz) v = w(kTGW, (int64_t)r * cz + c) * w(kTLnInW, c); break;
    }
    w16[idx] = __float2half_rn(v);
  }
  // Biases: b + W beta (f64 sums), padded with zeros; one warp per entry, lanes splitting the sum.
  const int lane = threadIdx.x & 31;
  for (int wi = (blockIdx.x * blockDim.x + threadIdx.x) >> 5; wi < kVecCount * C; wi += stride >> 5) {
    const int q = wi / C, e = wi % C;
    int tw = -1, tb = 0, tbeta = 0;
    int rows = 0, cols = 0;
    switch (q) {
      case kVBAP: tw = kTApW; tb = kTApB; tbeta = kTLnInB; rows = ch; cols = cz; break;
      case kVBAG: tw = kTAgW; tb = kTAgB; tbeta = kTLnInB; rows = ch; cols = cz; break;
      case kVBBP: tw = kTBpW; tb = kTBpB; tbeta = kTLnInB; rows = ch; cols = cz; break;
      case kVBBG: tw = kTBgW; tb = kTBgB; tbeta = kTLnInB; rows = ch; cols = cz; break;
      case kVBZ: tw = kTZW; tb = kTZB; tbeta = kTLnOutB; rows = cz; cols = ch; break;
      case kVBG: tw = kTGW; tb = kTGB; tbeta = kTLnInB; rows = cz; cols = cz; break;
      default: break;  // the LayerNorm slots are not used by the kernels
    }
    if (q == kVZSum) {  // the same rounded values the matrix holds
      tw = kTZW;
      rows = cz;
      cols = ch;
    }
    const bool live = tw >= 0 && e < rows;
    double acc = 0.0;
    if (live && q == kVZSum)
      for (int k = lane; k < cols; k += 32)
        acc += (double)__half2float(__float2half_rn(w(tw, (int64_t)e * cols + k) * w(kTLnOutW, k)));
    else if (live)
      for (int k = lane; k < cols; k += 32) acc += (double)w(tw, (int64_t)e * cols + k) * (double)w(tbeta, k);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
    if (lane == 0) vec[wi] = live ? static_cast<float>(acc + (q == kVZSum ? 0.0 : (double)w(tb, e))) : 0.f;
  }
}

// Offsets of the 16 tensors in the packed array (src/triangle/weights.ts:4-10).
static PackedAccess packed_access(const float *packed, int64_t cz, int64_t ch) {
  const int64_t sizes[kTensorCount] = {cz, cz, ch * cz, ch, ch * cz, ch, ch * cz, ch, ch * cz, ch, ch, ch,
                                       cz * ch, cz, cz * cz, cz};
  PackedAccess a{};
  a.packed = packed;
  int64_t off = 0;
  for (int t = 0; t < kTensorCount; ++t) {
    a.offset[t] = off;
    off += sizes[t];
  }
  return a;
}

// z [pairs][cz] (any dtype) -> f16 [pairs][128], zero-padded channels.
template <typename T>
__global__ void pad_z_kernel(const T *__restrict__ z, int64_t pairs, int cz, __half *__restrict__ z16) {
  const int64_t total = pairs * C;
  for (int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t p = idx / C;
    const int c = static_cast<int>(idx % C);
    z16[idx] = c < cz ? __float2half_rn(to_f32<T>(z[p * cz + c])) : __float2half_rn(0.f);
  }
}

// Loads a [128][128] f16 row-major matrix into two 128B-swizzled K chunks.
__device__ __forceinline__ void load_weight_matrix(uint8_t *dst, const __half *src, int tid, int nthreads) {
  for (int q = tid; q < C * 16; q += nthreads) {
    const int row = q >> 4, c16 = q & 15;
    const uint4 v = *reinterpret_cast<const uint4 *>(src + row * C + c16 * 8);
    *reinterpret_cast<uint4 *>(dst + (c16 >> 3) * 16384 + sw128_offset(row, c16 & 7)) = v;
  }
}

// ---------------------------------------------------------------------------
// Kernel 1: fused LayerNorm + gated projections.
// ---------------------------------------------------------------------------
constexpr int PJ_TILE = 64;      // pairs per tile
constexpr int PJ_STAGES = 3;
// warp 0 TMA, 1 MMA, 2-5 LayerNorm (every tile, two threads per pair row),
// 6-9 epilogue of a, 10-13 epilogue of b.
constexpr int PJ_THREADS = 448;
constexpr uint32_t PJ_CHUNK = PJ_TILE * 128;            // one 64-channel K chunk: 8 KB
constexpr uint32_t PJ_STAGE_BYTES = 2 * PJ_CHUNK;       // 16 KB
constexpr uint32_t PJ_W_BYTES = 4 * 2 * 16384;          // 128 KB
constexpr uint32_t PJ_OFF_STAGE = PJ_W_BYTES;
// Mask ring: each tile's 64 mask values, copied in by the producer warp and
// read by the epilogue (a ring of its own: the z stage is refilled before the
// epilogue of its tile runs).
constexpr int PJ_MASK_SLOTS = 4;
constexpr uint32_t PJ_OFF_MASK = PJ_OFF_STAGE + PJ_STAGES * PJ_STAGE_BYTES;
// Output staging: the tile's gated a and b, each [128 h][64 pairs] f16 in
// 128B-swizzled rows, written to HBM by two TMA stores.
constexpr uint32_t PJ_OFF_OUT = PJ_OFF_MASK + 2048;  // PJ_MASK_SLOTS x 64 f32 (1 KB), rounded up
constexpr uint32_t PJ_OUT_BYTES = 128 * 128;
constexpr uint32_t PJ_OFF_BAR = PJ_OFF_OUT + 2 * PJ_OUT_BYTES;
constexpr uint32_t PJ_SMEM = PJ_OFF_BAR + 256 + 1024;

struct ProjectArgs {
  const float *mask;
  int64_t mask_rs, mask_ks;  // mask of tile row r, pair k: mask[r * mask_rs + k * mask_ks]
  const __half *w16;
  const float *vec;
  int k_extent;              // pairs k per tile row (n, or this rank's rows for a sharded incoming product)
  int r_begin;               // first tile row of this launch (tile t covers row r_begin + t / tiles_k)
  int cz, tiles_k, total_tiles;
  int transposed;  // incoming: the z map is [k][j][c] and the box walks k in its outer dimension
  float eps;
  int store_maps;  // 1: one store per operand (box of all groups); R: one per channel group
  int hq;          // channels per group
  unsigned int *err;
};

// Where the gated operands go: map 0 covers all channel groups of this rank's operand buffer,
// or map g covers group g alone (in the buffer of the rank that contracts it: a peer's scratch
// mapped into this process, or this rank's own buffer for its own group).
constexpr int kMaxStoreMaps = 8;
struct ProjectStoreMaps {
  CUtensorMap a[kMaxStoreMaps], b[kMaxStoreMaps];
};

// Normalisation of pair row `row` of a 128B-swizzled K-major tile (two
// 64-channel chunks `chunk_bytes` apart), in place, 16-bit input -> f16:
// (x - mean) * rstd, with two threads per row: thread `half` takes the
// 64-channel chunk `half`; the pair combines its shifted sums with lane ^ 16
// (a warp holds 16 rows, so the 8 lanes of a quarter-warp read 8 different
// rows: no bank conflicts).  The LayerNorm's gamma and beta are folded into
// the weights that consume the tile.  Channels >= cz are padding (zero input)
// and stay out of the statistics.  The statistics are one pass over values
// shifted by the row's first channel (both threads use it), which keeps the
// f32 sums well conditioned.
template <typename ZT>
__device__ __forceinline__ void ln_row_pair(uint8_t *tile, uint32_t chunk_bytes, int row, int half, int cz,
                                            float inv_cz, float eps) {
  uint8_t *chunk = tile + half * chunk_bytes;
  const float x0 = unpack2<ZT>(*reinterpret_cast<const uint32_t *>(tile + sw128_offset(row, 0))).x;
  const float2 neg_x0 = f2(-x0);
  float2 s1 = f2(0.f), s2 = f2(0.f);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const uint4 v = *reinterpret_cast<const uint4 *>(chunk + sw128_offset(row, c));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 d = f2add(unpack2<ZT>(w[i]), neg_x0);
      if (cz != 128) {
        const int ch = half * 64 + c * 8 + 2 * i;
        d.x = ch < cz ? d.x : 0.f;
        d.y = ch + 1 < cz ? d.y : 0.f;
      }
      s1 = f2add(s1, d);
      s2 = f2fma(d, d, s2);
    }
  }
  float a1 = s1.x + s1.y, a2 = s2.x + s2.y;
  a1 += __shfl_xor_sync(kFull, a1, 16);
  a2 += __shfl_xor_sync(kFull, a2, 16);
  const float m1 = a1 * inv_cz;
  const float mean = x0 + m1;
  const float var = fmaxf(a2 * inv_cz - m1 * m1, 0.f);
  const float rstd = rsqrtf(var + eps);
  const float2 r2 = f2(rstd), sh2 = f2(-mean * rstd);
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    uint8_t *ptr = chunk + sw128_offset(row, c);
    const uint4 v = *reinterpret_cast<const uint4 *>(ptr);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 y = f2fma(unpack2<ZT>(w[i]), r2, sh2);
      o[i] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4 *>(ptr) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

template <typename ZT>
__global__ void __launch_bounds__(PJ_THREADS, 1)
    project_kernel(const __grid_constant__ CUtensorMap zmap, const __grid_constant__ ProjectStoreMaps smaps,
                   const ProjectArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + PJ_OFF_BAR;
  // barriers: z_full[3] z_ready[3] z_empty[3] acc_full[2] acc_empty[2] drain
  auto z_full = [&](int s) { return bar0 + 8u * s; };
  auto z_ready = [&](int s) { return bar0 + 8u * (3 + s); };
  auto z_empty = [&](int s) { return bar0 + 8u * (6 + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (9 + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (11 + b); };
  const uint32_t drain = bar0 + 8u * 13;
  const uint32_t out_full = bar0 + 8u * 14;  // all 8 epilogue warps have staged the tile
  const uint32_t out_free = bar0 + 8u * 15;  // the staged tile has been read by the TMA stores
  auto mask_full = [&](int m) { return bar0 + 8u * (16 + m); };   // a tile's mask has landed
  auto mask_empty = [&](int m) { return bar0 + 8u * (20 + m); };  // the epilogue has read it
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + PJ_OFF_BAR + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + PJ_OFF_BAR + 200);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;

  for (int m = 0; m < 4; ++m)
    load_weight_matrix(smem + m * 32768, p.w16 + (size_t)m * C * C, threadIdx.x, PJ_THREADS);
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < PJ_STAGES; ++s) {
      mbar_init(z_full(s), 1);
      mbar_init(z_ready(s), 4);
      mbar_init(z_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);
    }
    mbar_init(drain, 1);
    mbar_init(out_full, 8);
    mbar_init(out_free, 1);
    for (int m = 0; m < PJ_MASK_SLOTS; ++m) {
      mbar_init(mask_full(m), 32);
      mbar_init(mask_empty(m), 8);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer: lane 0 issues the z tiles by TMA, every lane copies two of the
    //      tile's 64 mask values (cp.async, zero past the extent) ----
    if (lane == 0) tma_prefetch_map(&zmap);
    int it = 0;
    int tr = blockIdx.x / p.tiles_k, tk = blockIdx.x % p.tiles_k;  // tile t = tr tiles_k + tk
    const int dr = gridDim.x / p.tiles_k, dk = gridDim.x % p.tiles_k;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int s = it % PJ_STAGES, m = it % PJ_MASK_SLOTS;
      const uint32_t ph = (it / PJ_STAGES) & 1;
      if (!warp_wait(z_empty(s), ph ^ 1, abort_flag, p.err, kErrWaitProducer) ||
          !warp_wait(mask_empty(m), ((it / PJ_MASK_SLOTS) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer))
        break;
      const int r = p.r_begin + tr, kb = tk;
      if (lane == 0) {
        const uint32_t dst = sbase + PJ_OFF_STAGE + s * PJ_STAGE_BYTES;
        mbar_arrive_expect_tx(z_full(s), PJ_STAGE_BYTES);
        const int c1 = p.transposed ? r : kb * PJ_TILE, c2 = p.transposed ? kb * PJ_TILE : r;
        tma_load_3d(dst, &zmap, z_full(s), 0, c1, c2);
        tma_load_3d(dst + PJ_CHUNK, &zmap, z_full(s), 64, c1, c2);
      }
      const uint32_t mdst = sbase + PJ_OFF_MASK + m * 256;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int k = kb * PJ_TILE + hh * 32 + lane;
        const bool valid = k < p.k_extent;
        const float *src = valid ? p.mask + (int64_t)r * p.mask_rs + (int64_t)k * p.mask_ks : p.mask;
        cp_async_4(mdst + (hh * 32 + lane) * 4, src, valid);
      }
      cp_async_arrive_noinc(mask_full(m));
      tk += dk;
      tr += dr;
      if (tk >= p.tiles_k) {
        tk -= p.tiles_k;
        ++tr;
      }
    }
    // every load issued has landed before the CTA exits (immediate unless a consumer gave up)
    cp_async_wait_all();
    if (lane == 0)
      for (int j = it > PJ_STAGES ? it - PJ_STAGES : 0; j < it; ++j)
        mbar_wait_drain(z_full(j % PJ_STAGES), (j / PJ_STAGES) & 1, p.err);
  } else if (warp == 1) {
    // ---- MMA issuer: the whole warp runs the loop, one elected lane issues ----
    constexpr uint32_t kIdesc = idesc_f16_f32(128, PJ_TILE);
    const uint64_t w_base = sdesc_k_sw128(sbase), z_base = sdesc_k_sw128(sbase + PJ_OFF_STAGE);
    int s = 0, buf = 0;
    uint32_t ph = 0, bph = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      if (!warp_wait(acc_empty(buf), bph ^ 1, abort_flag, p.err, kErrWaitMma) ||
          !warp_wait(z_ready(s), ph, abort_flag, p.err, kErrWaitMma))
        break;
      tc_fence_after();
      const uint64_t zd = z_base + s * (PJ_STAGE_BYTES >> 4);
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        const uint32_t d = tmem + buf * 256 + m * PJ_TILE;
#pragma unroll
        for (int kc = 0; kc < 2; ++kc) {
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) {
            const uint64_t ad = w_base + (((m * 2 + kc) * 16384 + ks * 32) >> 4);
            const uint64_t bd = zd + ((kc * PJ_CHUNK + ks * 32) >> 4);
            if (kc == 0 && ks == 0)
              umma_first(d, ad, bd, kIdesc);
            else
              umma_acc(d, ad, bd, kIdesc);
          }
        }
      }
      umma_commit(z_empty(s));
      umma_commit(acc_full(buf));
      if (++s == PJ_STAGES) {
        s = 0;
        ph ^= 1;
      }
      buf ^= 1;
      if (buf == 0) bph ^= 1;
    }
    // Every MMA has completed before TMEM is freed, whether or not a consumer gave up.
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else if (warp < 6) {
    // ---- LayerNorm of the z tile, in place, 16-bit -> f16 (every tile, in order) ----
    const int row = (warp - 2) * 16 + (lane & 15), half = lane >> 4;
    const float inv_cz = 1.f / static_cast<float>(p.cz);
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int s = it % PJ_STAGES;
      const uint32_t ph = (it / PJ_STAGES) & 1;
      if (!warp_wait(z_full(s), ph, abort_flag, p.err, kErrWaitNormalizer)) break;
      ln_row_pair<ZT>(smem + PJ_OFF_STAGE + s * PJ_STAGE_BYTES, PJ_CHUNK, row, half, p.cz, inv_cz, p.eps);
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(z_ready(s));
    }
  } else {
    // ---- epilogue: TMEM -> gated f16 operand rows, staged, stored by TMA ----
    const int e = warp - 6;        // 0..7
    const int op = e >> 2;         // 0: a (a_p, a_g), 1: b (b_p, b_g)
    const int q = warp & 3;        // TMEM lane quarter this warp may read
    // TMEM in the 16x256b shape: this thread takes channels h = 32 q + 8 ri + rq (ri = 0..3)
    // and the pair columns 8k + 2 cp, + 1 (k = 0..7), so it reads each pair's mask once for
    // four channels; each 4-byte pair is staged at its place in the channel's swizzled row.
    const int rq = lane >> 2, cp = lane & 3;
    const bool storer = e == 0 && lane == 0;
    bool store_pending = false;  // storer: a committed store may still be reading the staging buffer
    float2 gate_shift[4], bias_p2[4];
#pragma unroll
    for (int ri = 0; ri < 4; ++ri) {
      const int h = q * 32 + 8 * ri + rq;
      gate_shift[ri] = f2(0.5f * p.vec[(op ? kVBBG : kVBAG) * C + h]);
      bias_p2[ri] = f2(p.vec[(op ? kVBBP : kVBAP) * C + h]);
    }
    const float2 half2f = f2(0.5f);
    uint8_t *stage_op = smem + PJ_OFF_OUT + op * PJ_OUT_BYTES;
    int tr = blockIdx.x / p.tiles_k, tk = blockIdx.x % p.tiles_k;  // tile t = tr tiles_k + tk
    const int dr = gridDim.x / p.tiles_k, dk = gridDim.x % p.tiles_k;
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int r = p.r_begin + tr, k0 = tk * PJ_TILE;
      tk += dk;
      tr += dr;
      if (tk >= p.tiles_k) {
        tk -= p.tiles_k;
        ++tr;
      }
      const int buf = it & 1, m = it % PJ_MASK_SLOTS;
      const uint32_t bph = (it >> 1) & 1;
      const float *msk = reinterpret_cast<const float *>(smem + PJ_OFF_MASK + m * 256);
      if (!warp_wait(acc_full(buf), bph, abort_flag, p.err, kErrWaitEpilogue) ||
          !warp_wait(mask_full(m), (it / PJ_MASK_SLOTS) & 1, abort_flag, p.err, kErrWaitEpilogue))
        break;
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * 256 + op * 2 * PJ_TILE;
      // The whole tile leaves TMEM first and stays in registers as packed f16, so the
      // accumulator is released early and the previous tile's TMA store keeps reading the
      // staging buffer meanwhile.
      uint32_t pk[8][4];  // [k][ri]: pairs 8k + 2cp, + 1 of channel 32 q + 8 ri + rq
#pragma unroll
      for (int k = 0; k < PJ_TILE / 8; ++k) {
        const float2 mm = *reinterpret_cast<const float2 *>(msk + 8 * k + 2 * cp);
        uint32_t vp[2][4], vg[2][4];
#pragma unroll
        for (int g = 0; g < 2; ++g) {
          const uint32_t ga = taddr + (static_cast<uint32_t>(16 * g) << 16) + 8 * k;
          tmem_ld_16x256b_x1(ga, vp[g]);
          tmem_ld_16x256b_x1(ga + PJ_TILE, vg[g]);
        }
        tmem_ld_wait();
#pragma unroll
        for (int ri = 0; ri < 4; ++ri) {
          const int g = ri >> 1, hh = ri & 1;
          // a = mask (p + b_p) sigmoid(g + b_g), sigmoid(x) = 0.5 + 0.5 tanh(x / 2)
          const float2 arg =
              f2fma(make_float2(__uint_as_float(vg[g][2 * hh]), __uint_as_float(vg[g][2 * hh + 1])), half2f, gate_shift[ri]);
          const float2 sg = f2fma(make_float2(tanhf_approx(arg.x), tanhf_approx(arg.y)), half2f, half2f);
          const float2 pb =
              f2add(make_float2(__uint_as_float(vp[g][2 * hh]), __uint_as_float(vp[g][2 * hh + 1])), bias_p2[ri]);
          const float2 y = f2mul(f2mul(pb, sg), mm);
          pk[k][ri] = pack_half2(y.x, y.y);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(acc_empty(buf));
        mbar_arrive(mask_empty(m));
      }
      if (storer && store_pending) {  // the previous tile's stores have read the staging buffer
        bulk_wait_read_all();
        mbar_arrive(out_free);
        store_pending = false;
      }
      if (!warp_wait(out_free, (it & 1) ^ 1, abort_flag, p.err, kErrWaitEpilogue)) break;
      // 64 pairs = the eight 16-byte chunks of each channel's staged row; this thread's 4 bytes
#pragma unroll
      for (int ri = 0; ri < 4; ++ri) {
        const int h = q * 32 + 8 * ri + rq;
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<uint32_t *>(stage_op + h * 128 + ((k ^ (h & 7)) << 4) + 4 * cp) = pk[k][ri];
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(out_full);
      if (storer) {
        // both operand tiles staged: one TMA store each ([128 h] x 64 pairs of row r; with
        // channel shards the box's outer dimension scatters the groups of 128 / ranks channels)
        if (!mbar_wait(out_full, it & 1, abort_flag, p.err, kErrWaitEpilogue)) {
          it = -1;
        } else {
          if (p.store_maps == 1) {
            tma_store_4d(&smaps.a[0], sbase + PJ_OFF_OUT, k0, 0, r, 0);
            tma_store_4d(&smaps.b[0], sbase + PJ_OFF_OUT + PJ_OUT_BYTES, k0, 0, r, 0);
          } else {
            // group g's hq staged rows start g hq x 128 bytes in (a multiple of 1024: the
            // swizzle pattern is the whole block's)
            for (int g = 0; g < p.store_maps; ++g) {
              const uint32_t off = static_cast<uint32_t>(g * p.hq) * 128u;
              tma_store_4d(&smaps.a[g], sbase + PJ_OFF_OUT + off, k0, 0, r, 0);
              tma_store_4d(&smaps.b[g], sbase + PJ_OFF_OUT + PJ_OUT_BYTES + off, k0, 0, r, 0);
            }
          }
          bulk_commit();
          store_pending = true;
        }
      }
      if (__shfl_sync(kFull, it, 0) < 0) break;
    }
    if (storer) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
// ---------------------------------------------------------------------------
// Kernel 2: per-channel contraction X[h] = s * A[h] B[h]^T, on CTA pairs.
// ---------------------------------------------------------------------------
// A cluster of two CTAs computes a 256 x 256 tile of one channel with M = 256
// tcgen05 MMAs (cta_group::2): CTA r holds rows 128 r .. 128 r + 127 of the
// tile's A and of its B, so an SM reads 8 KB of operands per 128 x 256 x 16
// step (12 KB with one-CTA 128 x 256 tiles) and a third fewer operand bytes
// cross from L2.  Each CTA's TMEM receives its 128 rows (two 256-column
// accumulators, so the epilogue of one tile overlaps the MMAs of the next);
// the even CTA issues every MMA; the loads of both CTAs complete on its
// barriers.
constexpr int CT_BM = 128, CT_BN = 256, CT_BK = 64, CT_STAGES = 6, CT_THREADS = 192;
constexpr int CT_PAIR_M = 2 * CT_BM;                    // rows of a pair tile
constexpr uint32_t CT_A_BYTES = CT_BM * 128;             // this CTA's 128 rows of A per K block
constexpr uint32_t CT_B_BYTES = (CT_BN / 2) * 128;       // and its 128 rows of B
constexpr uint32_t CT_STAGE_BYTES = CT_A_BYTES + CT_B_BYTES;
// Epilogue staging: per epilogue warp two [32 rows][32 columns] f16 blocks (64B-swizzled rows),
// each written to the product by one TMA store.
constexpr uint32_t CT_OFF_XSTAGE = CT_STAGES * CT_STAGE_BYTES;
constexpr uint32_t CT_XSTAGE_BYTES = 2048;
constexpr uint32_t CT_OFF_BAR = CT_OFF_XSTAGE + 4 * 2 * CT_XSTAGE_BYTES;
constexpr uint32_t CT_SMEM = CT_OFF_BAR + 256 + 1024;

struct ContractArgs {
  __half *x_out;  // [row_count / block_rows_out][channels][block_rows_out][jp]
  int64_t x_hs, x_rs, x_bs;  // channel, row and block pitches of x_out
  int block_rows_out;        // product rows per block of x_out (one block unless channel-sharded)
  int n, row_begin, row_count;
  int k_split;               // k extent of one block of the operands' 4th map dimension
  // Channel-sharded: this rank's own share of the operands is read through the *_own maps
  // (own_mode 1: rows [own_row0, own_row0 + own_rows) of both operands; 2: k block own_kr),
  // and block own_blk of the product is written to x_own; so neither is copied.
  int own_mode, own_row0, own_rows, own_kr, own_blk;
  __half *x_own;
  int tiles_m, tiles_n, k_blocks, total_tiles;
  float scale;
  unsigned int *err;
};

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(CT_THREADS, 1)
    contract_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                    const __grid_constant__ CUtensorMap amap_own, const __grid_constant__ CUtensorMap bmap_own,
                    const __grid_constant__ CUtensorMap xmap_out, const __grid_constant__ CUtensorMap xmap_own,
                    const ContractArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + CT_OFF_BAR;
  // full: the leader's only (both CTAs' loads complete on it); empty, acc_full: both CTAs
  // (multicast commits); acc_empty: the leader's, one arrival per epilogue warp of the pair
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (CT_STAGES + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * CT_STAGES + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * CT_STAGES + 2 + b); };
  const uint32_t drain = bar0 + 8u * (2 * CT_STAGES + 4);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + CT_OFF_BAR + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + CT_OFF_BAR + 200);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_rank());
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_per_h = p.tiles_m * p.tiles_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < CT_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync_all();  // both CTAs' barriers exist before any arrival crosses the pair
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&amap);
      tma_prefetch_map(&bmap);
      int it = 0;
      bool ok = true;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        const int h = t / tiles_per_h, rem = t % tiles_per_h;
        const int mi = rem / p.tiles_n, ni = rem % p.tiles_n;
        int kl = 0, kr = 0;  // k = kr * k_split + kl: the operands may hold k in blocks (one per rank)
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % CT_STAGES;
          const uint32_t ph = (it / CT_STAGES) & 1;
          // the stage is free in this CTA once the pair's MMAs have read it (multicast commit)
          if (!mbar_wait(empty(s), ph ^ 1, abort_flag, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t dst = sbase + s * CT_STAGE_BYTES;
          if (leader) mbar_arrive_expect_tx(full(s), 2 * CT_STAGE_BYTES);
          const bool own_k = p.own_mode == 2 && kr == p.own_kr;
          auto own_row = [&](int row) {
            return p.own_mode == 1 && row >= p.own_row0 && row < p.own_row0 + p.own_rows;
          };
          const int arow = p.row_begin + mi * CT_PAIR_M + rank * CT_BM;
          if (own_k || own_row(arow))
            tma_load_4d_pair(dst, &amap_own, full(s), kl, h, own_k ? arow : arow - p.own_row0, 0);
          else
            tma_load_4d_pair(dst, &amap, full(s), kl, h, arow, kr);
          const int brow = ni * CT_BN + rank * (CT_BN / 2);
          if (own_k || own_row(brow))
            tma_load_4d_pair(dst + CT_A_BYTES, &bmap_own, full(s), kl, h, own_k ? brow : brow - p.own_row0, 0);
          else
            tma_load_4d_pair(dst + CT_A_BYTES, &bmap, full(s), kl, h, brow, kr);
          kl += CT_BK;
          if (kl >= p.k_split) {
            kl = 0;
            ++kr;
          }
        }
      }
      // every load issued has landed before the pair exits (the leader's barriers count
      // both CTAs' bytes; the peer waits for the leader at the final cluster barrier)
      if (leader)
        for (int j = it > CT_STAGES ? it - CT_STAGES : 0; j < it; ++j)
          mbar_wait_drain(full(j % CT_STAGES), (j / CT_STAGES) & 1, p.err);
    }
  } else if (warp == 1) {
    if (leader) {
      // the whole warp runs the issue loop (uniform waits, running descriptors); one elected lane issues
      constexpr uint32_t kIdesc = idesc_f16_f32(CT_PAIR_M, CT_BN);
      const uint64_t a_base = sdesc_k_sw128(sbase);  // stage s: + s * CT_STAGE_BYTES; B follows A
      uint64_t ad = a_base;
      int s = 0, buf = 0;
      uint32_t ph = 0, bph = 0;
      bool ok = true;
      for (int t = pair; t < p.total_tiles && ok; t += npairs) {
        if (!warp_wait(acc_empty(buf), bph ^ 1, abort_flag, p.err, kErrWaitMma)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * CT_BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!warp_wait(full(s), ph, abort_flag, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bd = ad + (CT_A_BYTES >> 4);
#pragma unroll
          for (int ks = 0; ks < CT_BK / 16; ++ks) umma_pair(d, ad + ks * 2, bd + ks * 2, kIdesc, (kb | ks) != 0);
          umma_commit_pair_both(empty(s));
          ad += CT_STAGE_BYTES >> 4;
          if (++s == CT_STAGES) {
            s = 0;
            ph ^= 1;
            ad = a_base;
          }
        }
        if (!ok) break;
        umma_commit_pair_both(acc_full(buf));
        buf ^= 1;
        if (buf == 0) bph ^= 1;
      }
      // Every MMA has completed before TMEM is freed, whether or not a consumer gave up.
      umma_commit_pair(drain);
      mbar_wait_drain(drain, 0, p.err);
    }
  } else {
    // Epilogue: each warp takes its TMEM lane quarter (32 product rows) in chunks of 32 columns:
    // TMEM -> scaled f16 -> a 64B-swizzled block in shared memory -> one TMA store into the
    // product (x_out, or x_own for this rank's own block), two blocks in flight per warp.
    const int q = warp & 3;
    const uint32_t stage0 = sbase + CT_OFF_XSTAGE + (warp - 2) * 2 * CT_XSTAGE_BYTES;
    uint8_t *stage0_ptr = smem + CT_OFF_XSTAGE + (warp - 2) * 2 * CT_XSTAGE_BYTES;
    int tile_it = 0, stores = 0;
    for (int t = pair; t < p.total_tiles; t += npairs, ++tile_it) {
      const int h = t / tiles_per_h, rem = t % tiles_per_h;
      const int mi = rem / p.tiles_n, ni = rem % p.tiles_n;
      const int buf = tile_it & 1;
      const uint32_t bph = (tile_it >> 1) & 1;
      if (!warp_wait(acc_full(buf), bph, abort_flag, p.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const int g0 = mi * CT_PAIR_M + rank * CT_BM + q * 32;  // the warp's first row inside this launch
      const bool rows_ok = g0 < p.row_count;
      const int blk = g0 / p.block_rows_out, gl0 = g0 - blk * p.block_rows_out;
      const bool own = blk == p.own_blk;
      const int j0 = ni * CT_BN;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * CT_BN;
#pragma unroll 1
      for (int chunk = 0; chunk < CT_BN / 32; ++chunk) {
        uint32_t v[32];
        tmem_ld32(taddr + chunk * 32, v);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2)
          pk[c >> 1] = pack_half2(__uint_as_float(v[c]) * p.scale, __uint_as_float(v[c + 1]) * p.scale);
        const int sb = stores & 1;
        if (lane == 0 && stores >= 2) bulk_wait_read_but_one();  // this block's previous store has read it
        __syncwarp();
        uint8_t *srow = stage0_ptr + sb * CT_XSTAGE_BYTES + lane * 64;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4 *>(srow + ((c ^ ((lane >> 1) & 3)) << 4)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
        fence_async_smem();
        __syncwarp();
        const int jc = j0 + chunk * 32;
        if (lane == 0 && rows_ok && jc < p.n) {  // rows and columns past the product are clipped
          const uint32_t src = stage0 + sb * CT_XSTAGE_BYTES;
          if (own)
            tma_store_3d(&xmap_own, src, jc, gl0, h);
          else
            tma_store_4d(&xmap_out, src, jc, gl0, h, blk);
        }
        if (lane == 0) bulk_commit();
        ++stores;
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_leader(acc_empty(buf));
    }
    if (lane == 0) bulk_wait_all();
  }

  tc_fence_before();
  cluster_sync_all();  // the pair's MMAs and loads are done before either CTA releases TMEM or exits
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Kernel 3: LN_out + output projection + gate + residual.
// ---------------------------------------------------------------------------
constexpr int OP_STAGES = 2;
// warp 0 TMA, 1 MMA, 2-5 LN_out statistics of X (two lanes per pair of pairs,
// each over half the channels), 6-13 LN_in of z (two threads per pair row),
// 14-21 epilogue (two warps per TMEM lane quarter: one thread per pair row and
// half of the 128 output channels).  Two warps per SM sub-partition in each
// of the z LayerNorm and the epilogue keep their dependent chains overlapped.
constexpr int OP_THREADS = 704;
constexpr uint32_t OP_W_BYTES = 2 * 2 * 16384;                 // W_z, W_g
constexpr uint32_t OP_X_BYTES = 128 * 256, OP_Z_BYTES = 128 * 256;
constexpr uint32_t OP_STAGE_BYTES = OP_X_BYTES + OP_Z_BYTES;
constexpr uint32_t OP_OFF_STAGE = OP_W_BYTES;
// Output staging for 16-bit outputs: [128 pairs][128 channels] as two
// 128B-swizzled halves of 64 channels, written by TMA (store or add).
constexpr uint32_t OP_OFF_OUT = OP_OFF_STAGE + OP_STAGES * OP_STAGE_BYTES;
constexpr uint32_t OP_OUT_BYTES = 128 * 256;
constexpr uint32_t OP_OFF_BAR = OP_OFF_OUT + OP_OUT_BYTES;
constexpr uint32_t OP_OFF_XSTAT = OP_OFF_BAR + 256;  // per pair (mean, rstd) of X: 128 float2
constexpr uint32_t OP_SMEM = OP_OFF_XSTAT + 1024 + 1024;

struct OutputArgs {
  void *out;
  int64_t out_rs;  // elements per pair row (c_z)
  const __half *w16;
  const float *vec;
  int n, cz, ch, row_begin, row_count, tiles_j, total_tiles, residual;
  float eps_in, eps_out;
  unsigned int *err;
};

template <typename ZT, typename OT>
__global__ void __launch_bounds__(OP_THREADS, 1)
    output_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap zmap,
                  const __grid_constant__ CUtensorMap omap, const OutputArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + OP_OFF_BAR;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto ready = [&](int s) { return bar0 + 8u * (2 + s); };
  auto empty = [&](int s) { return bar0 + 8u * (4 + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (6 + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (8 + b); };
  const uint32_t drain = bar0 + 8u * 10;
  const uint32_t out_full = bar0 + 8u * 11;  // all 4 epilogue warps have staged the tile
  const uint32_t out_free = bar0 + 8u * 12;  // the staged tile has been read by TMA
  const uint32_t stat_full = bar0 + 8u * 13;  // the X warps have written the tile's statistics
  const uint32_t stat_free = bar0 + 8u * 14;  // the epilogue warps have read them
  float2 *xstat = reinterpret_cast<float2 *>(smem + OP_OFF_XSTAT);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OP_OFF_BAR + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OP_OFF_BAR + 200);
  // Per-channel vectors are read straight from global memory: every lane of a
  // warp reads the same element, one broadcast through L1.
  const float *__restrict__ vbz = p.vec + kVBZ * C, *__restrict__ vbg = p.vec + kVBG * C;
  const float *__restrict__ vzs = p.vec + kVZSum * C;
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;
  const bool staged_out = sizeof(OT) == 2 && p.cz == C;

  load_weight_matrix(smem, p.w16 + (size_t)kWZ * C * C, threadIdx.x, OP_THREADS);
  load_weight_matrix(smem + 32768, p.w16 + (size_t)kWG * C * C, threadIdx.x, OP_THREADS);
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < OP_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(ready(s), 12);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 8);
    }
    mbar_init(drain, 1);
    mbar_init(out_full, 8);
    mbar_init(out_free, 1);
    mbar_init(stat_full, 4);
    mbar_init(stat_free, 8);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&xmap);
      tma_prefetch_map(&zmap);
      if (staged_out) tma_prefetch_map(&omap);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
        const int s = it % OP_STAGES;
        const uint32_t ph = (it / OP_STAGES) & 1;
        if (!mbar_wait(empty(s), ph ^ 1, abort_flag, p.err, kErrWaitProducer)) {
          ok = false;
          break;
        }
        const int il = t / p.tiles_j, j0 = (t % p.tiles_j) * 128;
        const uint32_t xs = sbase + OP_OFF_STAGE + s * OP_STAGE_BYTES, zs = xs + OP_X_BYTES;
        mbar_arrive_expect_tx(full(s), OP_STAGE_BYTES);
        tma_load_3d(xs, &xmap, full(s), j0, il, 0);
        tma_load_3d(xs + 16384, &xmap, full(s), j0 + 64, il, 0);
        tma_load_3d(zs, &zmap, full(s), 0, j0, p.row_begin + il);
        tma_load_3d(zs + 16384, &zmap, full(s), 64, j0, p.row_begin + il);
      }
      {  // every load issued has landed before the CTA exits (immediate unless a consumer gave up)
        for (int j = it > OP_STAGES ? it - OP_STAGES : 0; j < it; ++j)
          mbar_wait_drain(full(j % OP_STAGES), (j / OP_STAGES) & 1, p.err);
      }
    }
  } else if (warp == 1) {
    // the whole warp runs the issue loop (uniform waits, running descriptors); one elected lane issues
    constexpr uint32_t kIdesc = idesc_f16_f32(128, 128);
    constexpr uint32_t kIdescMn = idesc_f16_f32_amn(128, 128);
    const uint64_t x_base = sdesc_mn_sw128(sbase + OP_OFF_STAGE, 16384, 1024);
    const uint64_t z_base = sdesc_k_sw128(sbase + OP_OFF_STAGE + OP_X_BYTES);
    const uint64_t wz = sdesc_k_sw128(sbase), wg = sdesc_k_sw128(sbase + 32768);
    int s = 0, buf = 0;
    uint32_t ph = 0, bph = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      if (!warp_wait(acc_empty(buf), bph ^ 1, abort_flag, p.err, kErrWaitMma) ||
          !warp_wait(ready(s), ph, abort_flag, p.err, kErrWaitMma))
        break;
      tc_fence_after();
      const uint64_t xd = x_base + s * (OP_STAGE_BYTES >> 4), zd = z_base + s * (OP_STAGE_BYTES >> 4);
      const uint32_t d = tmem + buf * 256;
#pragma unroll
      for (int kc = 0; kc < 2; ++kc) {
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint32_t koff = (kc * 16384 + ks * 32) >> 4;
          // X is MN-major: K step (kc * 4 + ks) * 16 rows = that many 1024-byte atoms / 8 * 2.
          const uint64_t xk = xd + (((kc * 4 + ks) * 2048) >> 4);
          if (kc == 0 && ks == 0) {
            umma_first(d, xk, wz + koff, kIdescMn);
            umma_first(d + 128, zd + koff, wg + koff, kIdesc);
          } else {
            umma_acc(d, xk, wz + koff, kIdescMn);
            umma_acc(d + 128, zd + koff, wg + koff, kIdesc);
          }
        }
      }
      umma_commit(empty(s));
      umma_commit(acc_full(buf));
      if (++s == OP_STAGES) {
        s = 0;
        ph ^= 1;
      }
      buf ^= 1;
      if (buf == 0) bph ^= 1;
    }
    // Every MMA has completed before TMEM is freed, whether or not a consumer gave up.
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else if (warp < 14) {
    // ---- LN_out statistics of X (warps 2-5) and LN_in of z in place (warps 6-13) ----
    // X arrives MN-major: two 64-pair blocks 16 KB apart, each 128 h-rows of
    // 128 B, 128B-swizzled.  Lanes 2c and 2c + 1 of an X warp own the adjacent
    // pairs (2c', 2c' + 1) over the lower and upper half of the channels and
    // combine their shifted sums with one shuffle.  X is only read: the GEMM
    // consumes it as it landed, and the epilogue applies the statistics.
    const float inv_cz = 1.f / static_cast<float>(p.cz), inv_ch = 1.f / static_cast<float>(p.ch);
    const bool x_role = warp < 6;
    const int tx = (warp - 2) * 32 + lane;  // 0..127 among the X warps
    const int c = tx >> 1, hh = tx & 1;
    // z: a warp holds 16 rows, lanes l and l + 16 the two 64-channel halves of one
    const int zrow = (warp - 6) * 16 + (lane & 15), zhalf = lane >> 4;
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int s = it % OP_STAGES;
      const uint32_t ph = (it / OP_STAGES) & 1;
      if (!warp_wait(full(s), ph, abort_flag, p.err, kErrWaitNormalizer)) break;
      uint8_t *xs = smem + OP_OFF_STAGE + s * OP_STAGE_BYTES;
      uint8_t *zs = xs + OP_X_BYTES;
      if (x_role) {
        const int pair = 2 * c, mh = pair >> 6, pl = pair & 63;
        const uint8_t *col = xs + mh * 16384 + (pl & 7) * 2;
        auto word = [&](int h) {
          return *reinterpret_cast<const __half2 *>(col + h * 128 + ((((pl >> 3) ^ (h & 7))) << 4));
        };
        const float2 x0 = __half22float2(word(0));
        const float2 neg_x0 = make_float2(-x0.x, -x0.y);
        float2 s1 = f2(0.f), s2 = f2(0.f);
        // The upper half visits its rows in XOR-4 order within each group of
        // 8, so the two halves of a warp read disjoint banks.
        const int h0 = hh * 64, hx = hh * 4;
#pragma unroll 8
        for (int k = 0; k < 64; ++k) {
          const int h = h0 + (k ^ hx);
          float2 d = f2add(__half22float2(word(h)), neg_x0);
          if (p.ch != C && h >= p.ch) d = f2(0.f);
          s1 = f2add(s1, d);
          s2 = f2fma(d, d, s2);
        }
        // the stage's X has been read: the GEMM may go, the stage may be refilled after it
        fence_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(ready(s));
        s1.x += __shfl_xor_sync(kFull, s1.x, 1);
        s1.y += __shfl_xor_sync(kFull, s1.y, 1);
        s2.x += __shfl_xor_sync(kFull, s2.x, 1);
        s2.y += __shfl_xor_sync(kFull, s2.y, 1);
        const float2 m1 = f2mul(s1, f2(inv_ch));
        const float ra = rsqrtf(fmaxf(s2.x * inv_ch - m1.x * m1.x, 0.f) + p.eps_out);
        const float rb = rsqrtf(fmaxf(s2.y * inv_ch - m1.y * m1.y, 0.f) + p.eps_out);
        // the previous tile's statistics have been read by the epilogue
        if (it > 0 && !warp_wait(stat_free, (it - 1) & 1, abort_flag, p.err, kErrWaitNormalizer)) break;
        if (hh == 0) {
          xstat[pair] = make_float2(x0.x + m1.x, ra);
          xstat[pair + 1] = make_float2(x0.y + m1.y, rb);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(stat_full);
        continue;
      } else {
        ln_row_pair<ZT>(zs, 16384, zrow, zhalf, p.cz, inv_cz, p.eps_in);
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ready(s));
    }
  } else {
    // ---- epilogue: (LN_out(X) W_z^T + b_z) * sigmoid(LN(z) W_g^T + b_g) (+ residual) ----
    // LN_out(X) W_z'^T = rstd (D - mean rowsum(W_z')) with D = X W_z'^T from
    // the tensor core and the pair's (mean, rstd) from the X warps; the gate
    // is sigmoid(x) = 1/2 + tanh(x / 2) / 2.
    // 16-bit outputs with 128 channels are staged in shared memory and leave
    // through TMA: a plain store, or an add into the pair for the residual
    // form (the old values never pass through the SM).  Warps 14-17 take the
    // first 64 channels, 18-21 the second; in the staged form a thread owns
    // four pair rows and two of every eight of its half's channels (the 16x256b
    // TMEM shape), and the first half of them are computed into registers
    // before the staging buffer is claimed, so the previous tile's TMA keeps
    // reading it meanwhile.  Other outputs are written (and, for the residual,
    // read) by the thread that owns the row, one row and 64 channels each.
    const int q = warp & 3;
    const int pr = q * 32 + lane;
    const int cbase = ((warp - 14) >> 2) * 64;  // this thread's channels: cbase .. cbase + 63
    const bool storer = warp == 14 && lane == 0;
    bool store_pending = false;
    const float2 half2f = f2(0.5f);
    uint8_t *stage_row = smem + OP_OFF_OUT + pr * 128;
    float2 nmean2 = f2(0.f), rstd2 = f2(0.f);  // this pair row's LN_out statistics
    // The per-channel vectors of 8 channels c0 .. c0 + 7 (b_z, b_g / 2 and the
    // row sums of W_z'), loaded before the TMEM load they accompany: the TMEM
    // wait is a compiler barrier for memory accesses, so loads written after it
    // would only start once the accumulator has arrived.
    struct Vec8 {
      float4 bz[2], bg[2], zs[2];
    };
    auto load_vec8 = [&](int c0, Vec8 &v) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        v.bz[h] = *reinterpret_cast<const float4 *>(vbz + c0 + h * 4);
        v.bg[h] = *reinterpret_cast<const float4 *>(vbg + c0 + h * 4);
        v.zs[h] = *reinterpret_cast<const float4 *>(vzs + c0 + h * 4);
      }
    };
    // Output values of those 8 channels from their two accumulators, handed to
    // sink(cc, value pair of channels c0 + cc, c0 + cc + 1).
    auto gate8 = [&](const uint32_t (&vo)[8], const uint32_t (&vg)[8], const Vec8 &v, auto &&sink) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float2 bz2[2] = {make_float2(v.bz[h].x, v.bz[h].y), make_float2(v.bz[h].z, v.bz[h].w)};
        const float2 bg2[2] = {f2mul(make_float2(v.bg[h].x, v.bg[h].y), half2f),
                               f2mul(make_float2(v.bg[h].z, v.bg[h].w), half2f)};
        const float2 zs2[2] = {make_float2(v.zs[h].x, v.zs[h].y), make_float2(v.zs[h].z, v.zs[h].w)};
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int cc = h * 4 + 2 * i;
          const float2 arg = f2fma(make_float2(__uint_as_float(vg[cc]), __uint_as_float(vg[cc + 1])), half2f, bg2[i]);
          const float2 gate = f2fma(make_float2(tanhf_approx(arg.x), tanhf_approx(arg.y)), half2f, half2f);
          const float2 xo = f2fma(
              f2fma(zs2[i], nmean2, make_float2(__uint_as_float(vo[cc]), __uint_as_float(vo[cc + 1]))), rstd2, bz2[i]);
          sink(cc, f2mul(xo, gate));
        }
      }
    };
    // 8 channels c0.. as OT into the staged row: chunk (c0 % 64) / 8 of half c0 / 64.
    auto stage8 = [&](const uint4 &o, int c0) {
      uint8_t *half_row = stage_row + (c0 >> 6) * 16384;
      *reinterpret_cast<uint4 *>(half_row + ((((c0 & 63) >> 3) ^ (pr & 7)) << 4)) = o;
    };
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int il = t / p.tiles_j, j0 = (t % p.tiles_j) * 128, j = j0 + pr;
      const int buf = it & 1;
      const uint32_t bph = (it >> 1) & 1;
      if (!warp_wait(acc_full(buf), bph, abort_flag, p.err, kErrWaitEpilogue) ||
          !warp_wait(stat_full, it & 1, abort_flag, p.err, kErrWaitEpilogue))
        break;
      tc_fence_after();
      if (!staged_out) {
        const float2 st = xstat[pr];
        nmean2 = f2(-st.x);
        rstd2 = f2(st.y);
        __syncwarp();
        if (lane == 0) mbar_arrive(stat_free);
      }
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * 256;
      if (staged_out) {
        // TMEM in the 16x256b shape: this thread takes rows 16 g + 8 hh + rq of the quarter
        // (g, hh = 0, 1) and the channel pairs c = cbase + 8k + 2 cp, so it loads the three
        // per-channel vectors of two channels per k once for four rows; each 4-byte pair is
        // staged at its place in the 128B-swizzled row.
        const int rq = lane >> 2, cp = lane & 3;
        float nmean[4], rstdv[4];
#pragma unroll
        for (int ri = 0; ri < 4; ++ri) {
          const float2 st = xstat[q * 32 + 8 * ri + rq];
          nmean[ri] = -st.x;
          rstdv[ri] = st.y;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(stat_free);
        uint8_t *stage_half = smem + OP_OFF_OUT + (cbase >> 6) * 16384;
        auto stage_pair = [&](int ri, int k, uint32_t v) {
          const int r = q * 32 + 8 * ri + rq;
          *reinterpret_cast<uint32_t *>(stage_half + r * 128 + ((k ^ (r & 7)) << 4) + 4 * cp) = v;
        };
        uint32_t held[4][4];  // k = 0..3, rows ri: held until the staging buffer is claimed
        bool ok = true;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = cbase + 8 * k + 2 * cp;
          const float2 bz2 = *reinterpret_cast<const float2 *>(vbz + c);
          const float2 bg2 = f2mul(*reinterpret_cast<const float2 *>(vbg + c), half2f);
          const float2 zs2 = *reinterpret_cast<const float2 *>(vzs + c);
          uint32_t vo[2][4], vg[2][4];
#pragma unroll
          for (int g = 0; g < 2; ++g) {
            const uint32_t ga = taddr + (static_cast<uint32_t>(16 * g) << 16) + cbase + 8 * k;
            tmem_ld_16x256b_x1(ga, vo[g]);
            tmem_ld_16x256b_x1(ga + 128, vg[g]);
          }
          tmem_ld_wait();
          uint32_t out[4];
#pragma unroll
          for (int ri = 0; ri < 4; ++ri) {
            const int g = ri >> 1, hh = ri & 1;
            const float2 arg =
                f2fma(make_float2(__uint_as_float(vg[g][2 * hh]), __uint_as_float(vg[g][2 * hh + 1])), half2f, bg2);
            const float2 gate = f2fma(make_float2(tanhf_approx(arg.x), tanhf_approx(arg.y)), half2f, half2f);
            const float2 xo =
                f2fma(f2fma(zs2, f2(nmean[ri]), make_float2(__uint_as_float(vo[g][2 * hh]), __uint_as_float(vo[g][2 * hh + 1]))),
                      f2(rstdv[ri]), bz2);
            const float2 y = f2mul(xo, gate);
            out[ri] = pack2_t<OT>(y.x, y.y);
          }
          if (k < 4) {
#pragma unroll
            for (int ri = 0; ri < 4; ++ri) held[k][ri] = out[ri];
          } else {
            if (k == 4) {  // claim the staging buffer, then release the held channels into it
              if (storer && store_pending) {
                bulk_wait_read_all();
                mbar_arrive(out_free);
                store_pending = false;
              }
              ok = warp_wait(out_free, (it & 1) ^ 1, abort_flag, p.err, kErrWaitEpilogue);
              if (!ok) break;
#pragma unroll
              for (int kh = 0; kh < 4; ++kh)
#pragma unroll
                for (int ri = 0; ri < 4; ++ri) stage_pair(ri, kh, held[kh][ri]);
            }
#pragma unroll
            for (int ri = 0; ri < 4; ++ri) stage_pair(ri, k, out[ri]);
          }
        }
        if (!ok) break;
        fence_async_smem();
      } else {
        OT *orow = reinterpret_cast<OT *>(p.out) + ((int64_t)(p.row_begin + il) * p.n + j) * p.out_rs;
        const bool live = j < p.n;
#pragma unroll 1
        for (int part = 0; part < 8; ++part) {
          const int c0 = cbase + part * 8;
          Vec8 vec;
          load_vec8(c0, vec);
          uint32_t vo[8], vg[8];
          tmem_ld8(taddr + c0, vo);
          tmem_ld8(taddr + 128 + c0, vg);
          tmem_ld_wait();
          float v[8];
          gate8(vo, vg, vec, [&](int cc, float2 y) {
            v[cc] = y.x;
            v[cc + 1] = y.y;
          });
          if (live) {
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              if (c0 + cc < p.cz) {
                float x = v[cc];
                if (p.residual) x += to_f32<OT>(orow[c0 + cc]);
                orow[c0 + cc] = from_f32<OT>(x);
              }
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(acc_empty(buf));
        if (staged_out) mbar_arrive(out_full);
      }
      if (staged_out && storer) {
        if (!mbar_wait(out_full, it & 1, abort_flag, p.err, kErrWaitEpilogue)) {
          it = -1;
        } else {
          const int i = p.row_begin + il;
          if (p.residual) {
            tma_reduce_add_3d(&omap, sbase + OP_OFF_OUT, 0, j0, i);
            tma_reduce_add_3d(&omap, sbase + OP_OFF_OUT + 16384, 64, j0, i);
          } else {
            tma_store_3d(&omap, sbase + OP_OFF_OUT, 0, j0, i);
            tma_store_3d(&omap, sbase + OP_OFF_OUT + 16384, 64, j0, i);
          }
          bulk_commit();
          store_pending = true;
        }
      }
      if (__shfl_sync(kFull, it, 0) < 0) break;
    }
    if (staged_out && storer) bulk_wait_all();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}
}  // namespace tri

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------

TriangleLayout triangle_layout(int64_t n, int64_t cz, int64_t ch, int64_t block_rows, int z_dtype, int64_t rows,
                               int direction) {
  using tri::kChannelPad;
  TriangleLayout L;
  L.n = n;
  L.cz = cz;
  L.ch = ch;
  L.rows = (rows <= 0 || rows > n) ? n : rows;
  L.ranks = n / L.rows;
  L.hq = tri::C / L.ranks;
  const bool sharded = L.ranks > 1;
  L.block_rows = (!sharded && block_rows > 0 && block_rows < L.rows) ? block_rows : L.rows;
  // Projected operands [group][row][hq][k]: one group of hq channels per rank.  Outgoing:
  // rows i of this rank x all k; incoming: all rows j x this rank's k (its pair rows).
  const int64_t k_extent = (sharded && direction == AF2_INCOMING) ? L.rows : n;
  L.ab_rows = (sharded && direction == AF2_INCOMING) ? n : L.rows;
  L.kp = static_cast<int64_t>(align_up(static_cast<size_t>(k_extent), 8));
  L.jp = static_cast<int64_t>(align_up(static_cast<size_t>(n), 8));
  // Pitches are padded by 128 bytes so that rows and channel planes do not sit
  // an exact power of two apart (2^k-byte vectors times 2^k of them).
  L.ab_rs = L.hq * L.kp + kChannelPad;
  L.x_hs = L.block_rows * L.jp + kChannelPad;
  L.pad_z = (z_dtype == AF2_F32) || cz != tri::C;
  const size_t ab_bytes = sizeof(__half) * (size_t)L.ranks * L.ab_rows * L.ab_rs;
  const size_t x_bytes = sizeof(__half) * (size_t)tri::C * L.x_hs;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.off_w16 = take(sizeof(__half) * tri::kMatCount * tri::C * tri::C);
  L.off_vec = take(sizeof(float) * tri::kVecCount * tri::C);
  L.off_z16 = take(L.pad_z ? sizeof(__half) * (size_t)L.rows * n * tri::C : 0);
  // one GPU: a and b are [n][128][kp] (row-major, the contraction reads them in place)
  L.off_a = take(sharded ? ab_bytes : sizeof(__half) * (size_t)n * L.ab_rs);
  L.off_b = take(sharded ? ab_bytes : sizeof(__half) * (size_t)n * L.ab_rs);
  L.off_x = take(x_bytes);
  L.off_a_all = sharded ? take(ab_bytes) : L.off_a;
  L.off_b_all = sharded ? take(ab_bytes) : L.off_b;
  L.off_x_all = sharded ? take(x_bytes) : L.off_x;
  L.total = off;
  return L;
}

namespace {

// CTA pairs that can be resident at once for a cluster kernel (its __cluster_dims__
// of two): a persistent grid larger than this would leave pairs waiting for others to
// finish.  Returns 0 when the occupancy query fails, so that the caller uses a fallback
// for this launch only and asks again next time.
template <typename K>
int resident_pairs(af2_ctx *ctx, K kernel, int threads, uint32_t smem) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * std::max(1, ctx->sm_count / 2), 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &cfg) != cudaSuccess || clusters < 1) {
    cudaGetLastError();
    return 0;
  }
  return clusters;
}

CUtensorMapDataType map_type(int dtype) {
  return dtype == AF2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

template <typename ZT>
af2_status launch_project(af2_ctx *ctx, const CUtensorMap &zmap, const tri::ProjectStoreMaps &smaps,
                          const tri::ProjectArgs &a, cudaStream_t stream) {
  // set on every launch: the attribute belongs to the current device's copy of the kernel
  cudaError_t ce = cudaFuncSetAttribute(tri::project_kernel<ZT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        tri::PJ_SMEM);
  if (ce != cudaSuccess) return cuda_fail(ctx, ce, "configure project kernel");
  const int grid = std::max(1, std::min(a.total_tiles, ctx->sm_count));
  {
    LaunchScope scope(ctx, stream, kProfTriangleProject);
    tri::project_kernel<ZT><<<grid, tri::PJ_THREADS, tri::PJ_SMEM, stream>>>(zmap, smaps, a);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "launch project kernel");
}

template <typename ZT, typename OT>
af2_status launch_output(af2_ctx *ctx, const CUtensorMap &xmap, const CUtensorMap &zmap, const CUtensorMap &omap,
                         const tri::OutputArgs &a, cudaStream_t stream) {
  cudaError_t ce = cudaFuncSetAttribute(tri::output_kernel<ZT, OT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        tri::OP_SMEM);
  if (ce != cudaSuccess) return cuda_fail(ctx, ce, "configure output kernel");
  const int grid = std::max(1, std::min(a.total_tiles, ctx->sm_count));
  {
    LaunchScope scope(ctx, stream, kProfTriangleOutput);
    tri::output_kernel<ZT, OT><<<grid, tri::OP_THREADS, tri::OP_SMEM, stream>>>(xmap, zmap, omap, a);
  }
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "launch output kernel");
}

template <typename ZT>
af2_status launch_output_any(af2_ctx *ctx, int out_dtype, const CUtensorMap &xmap, const CUtensorMap &zmap,
                             const CUtensorMap &omap, const tri::OutputArgs &a, cudaStream_t stream) {
  switch (out_dtype) {
    case AF2_F32: return launch_output<ZT, float>(ctx, xmap, zmap, omap, a, stream);
    case AF2_F16: return launch_output<ZT, __half>(ctx, xmap, zmap, omap, a, stream);
    default: return launch_output<ZT, __nv_bfloat16>(ctx, xmap, zmap, omap, a, stream);
  }
}

}  // namespace

static int shard_rank(const TriangleShard *shard) { return shard ? shard->rank : 0; }

af2_status triangle_launch(af2_ctx *ctx, int direction, const TriangleLayout &L, const void *z, int z_dtype,
                           const float *mask, const float *packed, double eps, int residual, void *out,
                           int out_dtype, void *workspace, cudaStream_t stream, const TriangleShard *shard,
                           bool cache_weights, const af2_matrix *tensors) {
  using namespace tri;
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  // the prepared weights: the layout's prefix [0, off_z16), in the weight cache or the workspace
  WeightKey key;
  key.kind = kWeightsTriangle;
  key.ptr[0] = packed;
  key.dim[0] = L.cz;
  key.dim[1] = L.ch;
  if (tensors) {  // one tensor each: the key is their value arrays (the scales live beside them)
    key.kind = kWeightsTriangleTensors;
    for (int t = 0; t < kTensorCount; ++t) key.ptr[t] = tensors[t].values, key.ptr[16 + t] = tensors[t].scales;
  }
  PreparedRegion pw;
  if (af2_status st = prepared_region(ctx, key, L.off_z16, ws, cache_weights, &pw); st != AF2_OK) return st;
  __half *w16 = reinterpret_cast<__half *>(pw.base + L.off_w16);
  float *vec = reinterpret_cast<float *>(pw.base + L.off_vec);
  __half *a = reinterpret_cast<__half *>(ws + L.off_a);
  __half *b = reinterpret_cast<__half *>(ws + L.off_b);
  __half *x = reinterpret_cast<__half *>(ws + L.off_x);
  const int n = static_cast<int>(L.n);
  const int64_t rows = L.rows, R = L.ranks, hq = L.hq;
  const bool sharded = R > 1;
  if (sharded && (!shard || !shard->exchange || shard->ranks != R))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a row-sharded triangle multiplication needs the ranks' exchange");
  const int64_t pairs = rows * L.n;
  const bool out_dir = direction == AF2_OUTGOING;

  if (pw.fresh) {
    {
      LaunchScope scope(ctx, stream, kProfTrianglePrepare);
      if (tensors) {
        TensorAccess acc{};
        for (int t = 0; t < kTensorCount; ++t) {
          acc.values[t] = tensors[t].values;
          const bool q8 = tensors[t].format == AF2_WEIGHTS_Q8_BLOCK;
          acc.scales[t] = q8 ? static_cast<const uint16_t *>(tensors[t].scales) : nullptr;
          acc.block[t] = q8 ? tensors[t].block : 1;
        }
        prep_weights_kernel<<<96, 256, 0, stream>>>(acc, (int)L.cz, (int)L.ch, w16, vec);
      } else {
        prep_weights_kernel<<<96, 256, 0, stream>>>(packed_access(packed, L.cz, L.ch), (int)L.cz, (int)L.ch, w16,
                                                    vec);
      }
    }
    if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return cuda_fail(ctx, e, "launch weight preparation");
  }

  const void *zsrc = z;
  int zt = z_dtype;
  if (L.pad_z) {
    __half *z16 = reinterpret_cast<__half *>(ws + L.off_z16);
    const int grid = static_cast<int>(std::min<int64_t>((pairs * C + 255) / 256, 8 * 1024));
    LaunchScope scope(ctx, stream, kProfTriangleRelayout);
    switch (z_dtype) {
      case AF2_F32: pad_z_kernel<float><<<grid, 256, 0, stream>>>(static_cast<const float *>(z), pairs, (int)L.cz, z16); break;
      case AF2_F16: pad_z_kernel<__half><<<grid, 256, 0, stream>>>(static_cast<const __half *>(z), pairs, (int)L.cz, z16); break;
      default: pad_z_kernel<__nv_bfloat16><<<grid, 256, 0, stream>>>(static_cast<const __nv_bfloat16 *>(z), pairs, (int)L.cz, z16); break;
    }
    if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return cuda_fail(ctx, e, "launch z re-layout");
    zsrc = z16;
    zt = AF2_F16;
  }

  // ---- projections ----
  // Tile rows are pairs (r, k0..k0+63) outgoing and (k0..k0+63, r) incoming.  Both z maps
  // describe this rank's rows of z in their natural [row][col][c] order; the incoming box
  // is one column wide and 64 rows tall, which lands the same [64 rows][128 B] tile in
  // shared memory.  Outgoing: r runs over the local rows, k over all n; incoming: r over
  // all n columns, k over the local rows.
  const uint64_t row_bytes = C * 2;  // one pair row of the 128-channel z
  const int64_t r_extent = out_dir ? rows : L.n, k_extent = out_dir ? L.n : rows;
  CUtensorMap zmap_proj;
  if (!encode_map_3d(&zmap_proj, map_type(zt), zsrc, C, L.n, rows, row_bytes, row_bytes * L.n, 64,
                     out_dir ? PJ_TILE : 1, out_dir ? 1 : PJ_TILE, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the projection's z map");
  ProjectArgs pa;
  pa.mask = mask;  // this rank's rows [rows][n]
  pa.mask_rs = out_dir ? L.n : 1;
  pa.mask_ks = out_dir ? 1 : L.n;
  pa.w16 = w16;
  pa.vec = vec;
  pa.k_extent = static_cast<int>(k_extent);
  pa.cz = (int)L.cz;
  pa.tiles_k = static_cast<int>((k_extent + PJ_TILE - 1) / PJ_TILE);
  pa.r_begin = 0;
  pa.total_tiles = static_cast<int>(r_extent) * pa.tiles_k;
  pa.transposed = out_dir ? 0 : 1;
  pa.eps = static_cast<float>(eps);
  pa.err = ctx->err_word;
  // The gated operands leave through TMA stores into [group][row][hq][kp]: one box is 64 pairs
  // x 128 channels of one row, its outer dimension scattering the channel groups (one group
  // of all 128 channels on one GPU, so a row's channel vectors are contiguous there).
  const uint64_t ab_dims[4] = {(uint64_t)k_extent, (uint64_t)hq, (uint64_t)L.ab_rows, (uint64_t)R};
  const uint64_t ab_strides[3] = {(uint64_t)L.kp * 2, (uint64_t)L.ab_rs * 2, (uint64_t)L.ab_rows * L.ab_rs * 2};
  const uint32_t ab_box[4] = {PJ_TILE, (uint32_t)hq, 1, (uint32_t)R};
  ProjectStoreMaps smaps;
  std::memset(&smaps, 0, sizeof smaps);
  if (!encode_map_4d(&smaps.a[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a, ab_dims, ab_strides, ab_box,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_4d(&smaps.b[0], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, b, ab_dims, ab_strides, ab_box,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the projection's store maps");
  pa.store_maps = 1;
  pa.hq = static_cast<int>(hq);
  // ---- channel shards: every rank receives its hq channels of every rank's rows ----
  __half *a_all = reinterpret_cast<__half *>(ws + L.off_a_all), *b_all = reinterpret_cast<__half *>(ws + L.off_b_all);
  const size_t group_bytes = (size_t)L.ab_rows * L.ab_rs * sizeof(__half);
  const int me = shard_rank(shard);
  af2_status st = AF2_OK;
  // Direct exchange by copies (peer stores unavailable): the projection runs in two halves of
  // its tile rows (the rows of every channel group), and each half's groups are copied to their
  // ranks while the next computes.
  const bool direct = sharded && shard->direct && shard->direct(ctx, stream, &st);
  if (st != AF2_OK) return st;
  // With the peers' scratch mapped, channel group g leaves the projection by TMA store straight
  // into rank g's receive buffer (its slot for this rank), and this rank's own group into its
  // own buffer: no copies after the kernel.
  const bool peer_stores = direct && shard->peer_base && R <= kMaxStoreMaps && R > 1;
  // Before writing into the peers' receive buffers every peer must be done reading them.  The
  // shard scratch serves only this op, and the previous call ended with a barrier that every
  // rank passes only after its contraction (the reader of a and b) and whose output kernel (the
  // reader of X) precedes this call's projection barrier, so with peer stores no barrier is
  // needed here; the copy path keeps one.
  if (direct && !peer_stores && (st = shard->open(ctx, stream)) != AF2_OK) return st;
  if (peer_stores) {
    const uint64_t g_dims[4] = {(uint64_t)k_extent, (uint64_t)hq, (uint64_t)L.ab_rows, 1};
    const uint32_t g_box[4] = {PJ_TILE, (uint32_t)hq, 1, 1};
    const size_t slot = (size_t)me * group_bytes;
    for (int g = 0; g < R; ++g) {
      uint8_t *peer = g == me ? nullptr : static_cast<uint8_t *>(shard->peer_base(ctx, g));
      if (g != me && !peer) return fail(ctx, AF2_ERR_CUDA, "a peer's scratch is not mapped");
      const void *dst_a = g == me ? reinterpret_cast<uint8_t *>(a) + slot : peer + L.off_a_all + slot;
      const void *dst_b = g == me ? reinterpret_cast<uint8_t *>(b) + slot : peer + L.off_b_all + slot;
      if (!encode_map_4d(&smaps.a[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dst_a, g_dims, ab_strides, g_box,
                         CU_TENSOR_MAP_SWIZZLE_128B) ||
          !encode_map_4d(&smaps.b[g], CU_TENSOR_MAP_DATA_TYPE_FLOAT16, dst_b, g_dims, ab_strides, g_box,
                         CU_TENSOR_MAP_SWIZZLE_128B))
        return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the projection's peer store maps");
    }
    pa.store_maps = static_cast<int>(R);
  }
  const int64_t halves = (direct && !peer_stores && r_extent >= 2) ? 2 : 1, r_per = (r_extent + halves - 1) / halves;
  for (int64_t c = 0; c < halves; ++c) {
    const int64_t r0 = c * r_per, rc = std::min<int64_t>(r_per, r_extent - r0);
    pa.r_begin = static_cast<int>(r0);
    pa.total_tiles = static_cast<int>(rc) * pa.tiles_k;
    st = zt == AF2_BF16 ? launch_project<__nv_bfloat16>(ctx, zmap_proj, smaps, pa, stream)
                        : launch_project<__half>(ctx, zmap_proj, smaps, pa, stream);
    if (st != AF2_OK) return st;
    if (!direct || peer_stores) continue;
    // tile row r is row r of every channel group (outgoing: local pair row; incoming: column)
    const size_t off = (size_t)r0 * L.ab_rs * sizeof(__half), bytes = (size_t)rc * L.ab_rs * sizeof(__half);
    for (int64_t q = 1; q < R; ++q) {
      const int peer = static_cast<int>((me + q) % R);
      const size_t from = (size_t)peer * group_bytes + off, to = (size_t)me * group_bytes + off;
      if ((st = shard->send(ctx, reinterpret_cast<uint8_t *>(a) + from, reinterpret_cast<uint8_t *>(a_all) + to, bytes,
                            peer, stream)) != AF2_OK ||
          (st = shard->send(ctx, reinterpret_cast<uint8_t *>(b) + from, reinterpret_cast<uint8_t *>(b_all) + to, bytes,
                            peer, stream)) != AF2_OK)
        return st;
    }
  }
  // The contraction reads this rank's own share in place: its k block (incoming), or its
  // rows when they are whole 128-row tiles (outgoing); otherwise the share is copied over.
  const int own_mode = !sharded ? 0 : !out_dir ? 2 : rows % CT_BM == 0 ? 1 : 0;
  if (sharded) {
    if (direct) {
      if ((st = shard->close(ctx, stream)) != AF2_OK) return st;
    } else {
      const ShardTransfer ab[2] = {{a, a_all, group_bytes, group_bytes}, {b, b_all, group_bytes, group_bytes}};
      if ((st = shard->exchange(ctx, ab, 2, stream)) != AF2_OK) return st;
    }
    if (own_mode == 0) {
      const size_t at = (size_t)shard_rank(shard) * group_bytes;
      cudaError_t e = cudaMemcpyAsync(reinterpret_cast<uint8_t *>(a_all) + at, reinterpret_cast<uint8_t *>(a) + at,
                                      group_bytes, cudaMemcpyDeviceToDevice, stream);
      if (e == cudaSuccess)
        e = cudaMemcpyAsync(reinterpret_cast<uint8_t *>(b_all) + at, reinterpret_cast<uint8_t *>(b) + at, group_bytes,
                            cudaMemcpyDeviceToDevice, stream);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "own channel group copy");
    }
  }

  // ---- contraction maps: [k block][row][hq][k] viewed as {k, h, row, k block} ----
  // Outgoing: rows i of a x rows j of b, k over all n (one k block).  Incoming: rows i of b'
  // x rows j of a', k over n in one block per rank (each rank's pair rows), in k order.
  const __half *m_op = out_dir ? a_all : b_all;  // rows i of the product
  const __half *n_op = out_dir ? b_all : a_all;  // rows j of the product
  const int64_t op_rows = sharded ? L.n : (out_dir ? rows : L.n);
  const int64_t kblk = (sharded && !out_dir) ? rows : L.n, nkblk = (sharded && !out_dir) ? R : 1;
  const uint64_t m_dims[4] = {(uint64_t)kblk, (uint64_t)hq, (uint64_t)op_rows, (uint64_t)nkblk};
  const uint64_t n_dims[4] = {(uint64_t)kblk, (uint64_t)hq, (uint64_t)L.n, (uint64_t)nkblk};
  const uint64_t op_strides[3] = {(uint64_t)L.kp * 2, (uint64_t)L.ab_rs * 2, (uint64_t)L.n * L.ab_rs * 2};
  const uint32_t box[4] = {CT_BK, 1, CT_BM, 1};  // each CTA of a pair loads one A and one B box per K block
  // this rank's own share, read from the projected operands in place (not exchanged):
  // outgoing its rows, incoming its k block
  const size_t group = (size_t)L.ab_rows * L.ab_rs;
  const __half *m_own = (out_dir ? a : b) + (size_t)shard_rank(shard) * group;
  const __half *n_own = (out_dir ? b : a) + (size_t)shard_rank(shard) * group;
  const uint64_t own_dims[4] = {(uint64_t)kblk, (uint64_t)hq, (uint64_t)(out_dir ? rows : L.n), 1};
  CUtensorMap amap, bmap, amap_own, bmap_own, zmap_out;
  if (!encode_map_4d(&amap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, m_op, m_dims, op_strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_4d(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n_op, n_dims, op_strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_4d(&amap_own, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, m_own, own_dims, op_strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_4d(&bmap_own, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, n_own, own_dims, op_strides, box,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&zmap_out, map_type(zt), zsrc, C, L.n, rows, row_bytes, row_bytes * L.n, 64, 128, 1,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the contraction maps");
  // 16-bit outputs with 128 channels leave through TMA: [N][N][128], one box = 64 channels x 128 pairs.
  CUtensorMap omap;
  std::memset(&omap, 0, sizeof omap);
  if (out_dtype != AF2_F32 && L.cz == C &&
      !encode_map_3d(&omap, map_type(out_dtype), out, C, L.n, rows, row_bytes, row_bytes * L.n, 64, 128, 1,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the output store map");
  // the attribute is per device, so it is set for this context's device on every call; the
  // resident-pair count it allows is queried once per context
  if (cudaError_t e = cudaFuncSetAttribute(contract_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, CT_SMEM);
      e != cudaSuccess)
    return cuda_fail(ctx, e, "configure contraction kernel");
  // only a successful query is kept; after a failed one this launch uses half the SMs' worth of
  // pairs (a grid that may exceed what is resident, which costs time, not results)
  if (ctx->contract_pairs == 0) ctx->contract_pairs = resident_pairs(ctx, contract_kernel, CT_THREADS, CT_SMEM);
  const int contract_pairs = ctx->contract_pairs > 0 ? ctx->contract_pairs : std::max(1, ctx->sm_count / 2);
  auto contract = [&](int64_t rb, int64_t rc, int64_t rows_per_block, __half *x_base, int own_blk) -> af2_status {
    ContractArgs ca;
    ca.x_out = x_base;
    ca.x_hs = L.x_hs;
    ca.x_rs = L.jp;
    ca.x_bs = hq * L.x_hs;
    ca.block_rows_out = static_cast<int>(rows_per_block);
    ca.n = n;
    ca.row_begin = static_cast<int>(rb);
    ca.row_count = static_cast<int>(rc);
    ca.k_split = static_cast<int>(kblk);
    ca.own_mode = own_mode;
    ca.own_row0 = static_cast<int>(shard_rank(shard) * rows);
    ca.own_rows = static_cast<int>(rows);
    ca.own_kr = shard_rank(shard);
    ca.own_blk = own_blk;
    ca.x_own = reinterpret_cast<__half *>(ws + L.off_x_all) + (size_t)shard_rank(shard) * hq * L.x_hs;
    ca.tiles_m = static_cast<int>((rc + CT_PAIR_M - 1) / CT_PAIR_M);
    ca.tiles_n = (n + CT_BN - 1) / CT_BN;
    ca.k_blocks = (n + CT_BK - 1) / CT_BK;
    ca.total_tiles = static_cast<int>(hq) * ca.tiles_m * ca.tiles_n;
    ca.scale = 1.0f / static_cast<float>(n);
    ca.err = ctx->err_word;
    // product stores: [block][hq][rows_per_block][jp] (x_base) and this rank's own block, boxes of
    // 32 columns x 32 rows
    CUtensorMap xmap_out, xmap_own;
    std::memset(&xmap_own, 0, sizeof xmap_own);
    const uint64_t nblk = static_cast<uint64_t>((rc + rows_per_block - 1) / rows_per_block);
    const uint64_t xdims[4] = {static_cast<uint64_t>(n), static_cast<uint64_t>(rows_per_block),
                               static_cast<uint64_t>(hq), nblk};
    const uint64_t xstr[3] = {static_cast<uint64_t>(L.jp) * 2, static_cast<uint64_t>(L.x_hs) * 2,
                              static_cast<uint64_t>(hq * L.x_hs) * 2};
    const uint32_t xbox[4] = {32, 32, 1, 1};
    if (!encode_map_4d(&xmap_out, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, x_base, xdims, xstr, xbox,
                       CU_TENSOR_MAP_SWIZZLE_64B) ||
        (own_blk >= 0 && !encode_map_3d(&xmap_own, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ca.x_own, n, rows_per_block, hq,
                                        L.jp * 2, (uint64_t)L.x_hs * 2, 32, 32, 1, CU_TENSOR_MAP_SWIZZLE_64B)))
      return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the contraction's product maps");
    // CTA pairs: an even grid of at most the pairs that can be resident together
    const int grid = 2 * std::max(1, std::min(ca.total_tiles, contract_pairs));
    {
      LaunchScope scope(ctx, stream, kProfTriangleContract);
      contract_kernel<<<grid, CT_THREADS, CT_SMEM, stream>>>(amap, bmap, amap_own, bmap_own, xmap_out, xmap_own, ca);
    }
    const cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "launch contraction");
  };
  auto output = [&](const __half *xb, int64_t rb, int64_t rc) -> af2_status {
    CUtensorMap xmap;
    if (!encode_map_3d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xb, L.n, rc, C, L.jp * 2, (uint64_t)L.x_hs * 2, 64, 1,
                       C, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the contracted block");
    OutputArgs oa;
    oa.out = out;
    oa.out_rs = L.cz;
    oa.w16 = w16;
    oa.vec = vec;
    oa.n = n;
    oa.cz = (int)L.cz;
    oa.ch = (int)L.ch;
    oa.row_begin = static_cast<int>(rb);
    oa.row_count = static_cast<int>(rc);
    oa.tiles_j = (n + 127) / 128;
    oa.total_tiles = static_cast<int>(rc) * oa.tiles_j;
    oa.residual = residual;
    oa.eps_in = static_cast<float>(eps);
    oa.eps_out = static_cast<float>(eps / ((double)n * (double)n));
    oa.err = ctx->err_word;
    return zt == AF2_BF16 ? launch_output_any<__nv_bfloat16>(ctx, out_dtype, xmap, zmap_out, omap, oa, stream)
                          : launch_output_any<__half>(ctx, out_dtype, xmap, zmap_out, omap, oa, stream);
  };

  if (sharded) {
    // hq channels of every product row, written in one block per destination rank
    // ([rank][hq][rows][jp]); the exchange gathers all 128 channels of this rank's rows.
    __half *x_all = reinterpret_cast<__half *>(ws + L.off_x_all);
    const size_t xblock = (size_t)hq * L.x_hs * sizeof(__half);
    if (direct) {
      // one aligned group of destination row blocks at a time (a group spans at least one
      // 256-row pair tile, so blocks of 64 or 128 rows are not contracted as half-empty
      // tiles), the groups of peers first: each group's blocks leave while the next group is
      // contracted, and the group holding this rank's own block (written in place) comes last
      const int64_t per = std::min<int64_t>(R, (CT_PAIR_M + rows - 1) / rows), groups = R / per;
      for (int64_t q = 1; q <= groups; ++q) {
        const int64_t d0 = ((me / per + q) % groups) * per;
        __half *xb = reinterpret_cast<__half *>(reinterpret_cast<uint8_t *>(x) + (size_t)d0 * xblock);
        const int own = (me >= d0 && me < d0 + per) ? static_cast<int>(me - d0) : -1;
        if ((st = contract(d0 * rows, per * rows, rows, xb, own)) != AF2_OK) return st;
        for (int64_t d = d0; d < d0 + per; ++d) {
          if (d == me) continue;
          const uint8_t *src = reinterpret_cast<const uint8_t *>(x) + (size_t)d * xblock;
          if ((st = shard->send(ctx, src, reinterpret_cast<uint8_t *>(x_all) + (size_t)me * xblock, xblock,
                                static_cast<int>(d), stream)) != AF2_OK)
            return st;
        }
      }
      if ((st = shard->close(ctx, stream)) != AF2_OK) return st;
    } else if ((st = contract(0, L.n, rows, x, me)) != AF2_OK ||
               (st = shard->exchange(ctx, std::array<ShardTransfer, 1>{{{x, x_all, xblock, xblock}}}.data(), 1,
                                     stream)) != AF2_OK) {
      return st;
    }
    return output(x_all, 0, rows);
  }
  // one GPU: per block of output rows, contraction then output
  for (int64_t rb = 0; rb < rows; rb += L.block_rows) {
    const int64_t rc = std::min<int64_t>(L.block_rows, rows - rb);
    if ((st = contract(rb, rc, rc, x, -1)) != AF2_OK || (st = output(x, rb, rc)) != AF2_OK) return st;
  }
  return AF2_OK;
}

}  // namespace af2
