// transition.cu -- the Evoformer transition (LayerNorm -> Linear C->H -> ReLU
// -> Linear H->C, optional residual) as one persistent tcgen05 kernel, the
// weight preparation that turns f32 or mixed-q8 weights into its f16 operand
// tiles, and the bit-exact q8 decode.
//
// Reference: src/evoformer/transition.ts:91-138 (createLinearShader, the
// A W + b (ReLU) projection), :179-245 (the LayerNorm kernel), :264-361
// (TransitionGpu.run: normalise, first linear, second linear per row chunk)
// and src/evoformer/block.ts:625-740 (encodeTransition with residualTarget);
// q8 decode src/reference/dtype.ts:86-97.
//
// Kernel (one CTA per SM, 128-row tiles, persistent):
//   warp 0      TMA: the x tile (16-bit, straight into the first GEMM's A
//               operand) and the weight chunks through a 2-deep ring;
//   warp 1      tcgen05 issue over one continuous stream of 128-wide hidden
//               chunks j (all tiles of the CTA back to back): D1[j%2] =
//               xn W1[:, chunk], and one chunk behind it, D2[tile] +=
//               H[j-1] W2[chunk j-1, :] -- so the tensor pipe has the next
//               first-GEMM chunk queued while the epilogue turns a finished
//               one into the second GEMM's operand;
//   warps 2-5   row warps: LayerNorm of the next x tile in place (one
//               thread per row), then the second epilogue of this tile:
//               D2 -> scale2 * acc + b2, staged and written by per-warp TMA
//               stores (or TMA adds for the residual);
//   warps 6-13  first epilogue, two groups of four taking alternate chunks:
//               D1 -> relu(scale1 * acc + b1) as f16 into the second GEMM's
//               A operand (shared memory, never HBM).
// The hidden activations (4C per row) never leave the SM, so HBM traffic is
// one read of x and one write of the output.
//
// Weights: the kernel multiplies f16 operands.  Every output column o of a
// matrix carries an f32 scale applied in the epilogue: for per-channel q8 it
// is the given scale and the operand holds the int8 codes themselves (exact
// in f16); for f32 and block-q8 weights (decoded exactly to f32 first) it is
// a power of two that brings the column's largest magnitude into [0.5, 1),
// so the f16 rounding error is relative to the column's range.
#include <algorithm>
#include <string>

#include "af2_device.cuh"
#include "af2_internal.h"

namespace af2 {
namespace trn {

constexpr int TILE = 128;     // rows per tile (one TMEM lane each)
constexpr int HC = 128;       // hidden channels per chunk (the first GEMM's N)
constexpr int STAGES = 4;     // weight-chunk ring
constexpr int LAG = 1;        // second-GEMM chunks trail the first by this many
constexpr int NBUF = 2;       // D1 accumulators, each holding its H operand once converted (> LAG)
// 14 warps: 0 TMA, 1 MMA, 2-5 second epilogue, 6-9 LayerNorm of the x tiles, 10-13 first epilogue
constexpr int THREADS = 448;

// Shared-memory map (bytes from the 1024-aligned base); kb = channel blocks of 64.
//   A  2 x [kb][128 rows][128 B]      x tiles (normalised in place)
//   W  STAGES x kb x 16 KB            weight chunks: W1 [kb][128 h][128 B], W2 [2][cp][128 B]
//   O  [128 rows][128 B]              output staging (64 channels at a time)
// The relu(hidden) chunks (the second GEMM's A operand, f16) never reach shared
// memory: the first epilogue writes each into the first 64 TMEM columns of the
// D1 accumulator it came from, and the second GEMM reads A from TMEM.
//   barriers, then gamma beta scale2 bias2 [cp] and scale1 bias1 [hp]
__host__ __device__ constexpr uint32_t off_w(int kb) { return 2u * kb * 16384u; }
__host__ __device__ constexpr uint32_t off_o(int kb) { return off_w(kb) + STAGES * kb * 16384u; }
__host__ __device__ constexpr uint32_t off_bar(int kb) { return off_o(kb) + 16384u; }
__host__ __device__ constexpr uint32_t off_vec(int kb) { return off_bar(kb) + 512u; }

// Output modes.
enum { kOutTmaStore = 0, kOutTmaAdd = 1, kOutDirect = 2, kOutDirectAdd = 3 };

struct Args {
  const float *vec;  // gamma[cp] beta[cp] s1[hp] b1[hp] s2[cp] b2[cp]
  void *out;         // direct-store modes: [rows][c] of OT
  int64_t rows;
  int c, cp, kb, hp, nh, total_tiles;
  int normalize;  // 1: x is raw 16-bit, normalised in place; 0: x is already LayerNorm(x) in f16
  int out_mode;
  float eps;
  unsigned int *err;
};

// Position in a CTA's stream of hidden chunks without runtime divisions (the
// issuing threads are single threads on the critical path, where an integer
// division by nh costs more than the MMAs it schedules): tile `it` of the
// CTA, step `h` within the tile, and the hidden chunk that step covers.  Each
// tile starts its walk at chunk (tile index mod nh), so the CTAs do not all
// fetch the same weight chunk at the same moment; the order depends on the
// tile alone, so results do not depend on the grid.
struct ChunkCursor {
  int it = 0, h = 0, chunk = 0, nh = 1;
  __device__ __forceinline__ void start(int nh_) {
    nh = nh_;
    it = h = 0;
    chunk = static_cast<int>(blockIdx.x) % nh;
  }
  __device__ __forceinline__ void advance() {
    if (++h == nh) {
      h = 0;
      ++it;
      chunk = static_cast<int>((blockIdx.x + it * gridDim.x) % nh);
    } else if (++chunk == nh) {
      chunk = 0;
    }
  }
};

// LayerNorm of row `row` of a 128B-swizzled K-major tile ([kb][128 rows][128 B])
// in place, 16-bit in -> f16 out: (x - mean) * rstd * gamma + beta.  Channels
// >= c are zero padding: outside the statistics, and gamma = beta = 0 there.
// The sums run over values shifted by the row's first element, which keeps
// the single-pass f32 variance well conditioned.
template <typename XT>
__device__ __forceinline__ void ln_row(uint8_t *tile, int kb, int row, int c, float inv_c, float eps,
                                       const float *gamma, const float *beta) {
  auto chunk_ptr = [&](int j) { return tile + (j >> 3) * 16384 + sw128_offset(row, j & 7); };
  const int chunks = kb * 8;
  const float x0 = unpack2<XT>(reinterpret_cast<const uint32_t *>(chunk_ptr(0))[0]).x;
  const float2 neg_x0 = f2(-x0);
  float2 s1 = f2(0.f), s2 = f2(0.f);
#pragma unroll 4
  for (int j = 0; j < chunks; ++j) {
    const uint4 v = *reinterpret_cast<const uint4 *>(chunk_ptr(j));
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 d = f2add(unpack2<XT>(w[i]), neg_x0);
      const int ch = j * 8 + 2 * i;
      d.x = ch < c ? d.x : 0.f;
      d.y = ch + 1 < c ? d.y : 0.f;
      s1 = f2add(s1, d);
      s2 = f2fma(d, d, s2);
    }
  }
  const float m1 = (s1.x + s1.y) * inv_c;
  const float mean = x0 + m1;
  const float var = fmaxf((s2.x + s2.y) * inv_c - m1 * m1, 0.f);
  const float rstd = rsqrtf(var + eps);
  const float2 r2 = f2(rstd), nm2 = f2(-mean);
#pragma unroll 2
  for (int j = 0; j < chunks; ++j) {
    uint8_t *ptr = chunk_ptr(j);
    const uint4 v = *reinterpret_cast<const uint4 *>(ptr);
    const float4 g0 = *reinterpret_cast<const float4 *>(gamma + j * 8);
    const float4 g1 = *reinterpret_cast<const float4 *>(gamma + j * 8 + 4);
    const float4 b0 = *reinterpret_cast<const float4 *>(beta + j * 8);
    const float4 b1 = *reinterpret_cast<const float4 *>(beta + j * 8 + 4);
    const float2 g[4] = {make_float2(g0.x, g0.y), make_float2(g0.z, g0.w), make_float2(g1.x, g1.y),
                         make_float2(g1.z, g1.w)};
    const float2 b[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                         make_float2(b1.z, b1.w)};
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = f2mul(g[i], r2);              // rstd * gamma
      const float2 y = f2fma(f2add(unpack2<XT>(w[i]), nm2), a, b[i]);
      o[i] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4 *>(ptr) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// The same LayerNorm for tiles of two 64-channel blocks with four threads per
// row: thread `quarter` takes channels 32 quarter .. 32 quarter + 31 (block
// quarter / 2, 16-byte chunks 4 (quarter % 2) ..) and holds their gamma and
// beta in registers (g, b), so a tile costs no loads of them; the four combine
// their shifted sums with lanes ^ 8 and ^ 16.
template <typename XT>
__device__ __forceinline__ void ln_row_quad(uint8_t *tile, int row, int quarter, int c, float inv_c, float eps,
                                            const float2 (&g)[16], const float2 (&b)[16]) {
  uint8_t *blk = tile + (quarter >> 1) * 16384;
  const int c0 = (quarter & 1) * 4;
  const float x0 = unpack2<XT>(*reinterpret_cast<const uint32_t *>(tile + sw128_offset(row, 0))).x;
  const float2 neg_x0 = f2(-x0);
  float2 s1 = f2(0.f), s2 = f2(0.f);
  uint4 v[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) v[k] = *reinterpret_cast<const uint4 *>(blk + sw128_offset(row, c0 + k));
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float2 d = f2add(unpack2<XT>(w[i]), neg_x0);
      const int ch = quarter * 32 + k * 8 + 2 * i;
      d.x = ch < c ? d.x : 0.f;
      d.y = ch + 1 < c ? d.y : 0.f;
      s1 = f2add(s1, d);
      s2 = f2fma(d, d, s2);
    }
  }
  float a1 = s1.x + s1.y, a2 = s2.x + s2.y;
  a1 += __shfl_xor_sync(kFull, a1, 8);
  a2 += __shfl_xor_sync(kFull, a2, 8);
  a1 += __shfl_xor_sync(kFull, a1, 16);
  a2 += __shfl_xor_sync(kFull, a2, 16);
  const float m1 = a1 * inv_c;
  const float mean = x0 + m1;
  const float var = fmaxf(a2 * inv_c - m1 * m1, 0.f);
  const float rstd = rsqrtf(var + eps);
  const float2 r2 = f2(rstd), nm2 = f2(-mean);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
    uint32_t o[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 a = f2mul(g[4 * k + i], r2);  // rstd * gamma
      const float2 y = f2fma(f2add(unpack2<XT>(w[i]), nm2), a, b[4 * k + i]);
      o[i] = pack_half2(y.x, y.y);
    }
    *reinterpret_cast<uint4 *>(blk + sw128_offset(row, c0 + k)) = make_uint4(o[0], o[1], o[2], o[3]);
  }
}

// Two f32 -> packed f16 with ReLU (cvt.rn.relu: max(0, round(v)) = round(max(0, v))).
__device__ __forceinline__ uint32_t pack_half2_relu(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.relu.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename OT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float lo, float hi) {
  return pack_half2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<float>(float, float) {
  return 0;  // f32 output never goes through the 16-bit staging
}

template <typename XT, typename OT, int KB>
__global__ void __launch_bounds__(THREADS, 1)
    transition_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap w1map,
                      const __grid_constant__ CUtensorMap w2map, const __grid_constant__ CUtensorMap omap,
                      const Args p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  constexpr int kb = KB;
  const uint32_t OFF_W = off_w(kb), OFF_O = off_o(kb), OFF_BAR = off_bar(kb);
  const uint32_t A_BYTES = kb * 16384u, W_BYTES = kb * 16384u;
  const uint32_t W2_KSTRIDE = p.cp * 128u;  // bytes between the two 64-wide K blocks of a W2 chunk
  const uint32_t bar0 = sbase + OFF_BAR;
  auto a_raw = [&](int b) { return bar0 + 8u * b; };
  auto a_full = [&](int b) { return bar0 + 8u * (2 + b); };
  auto a_empty = [&](int b) { return bar0 + 8u * (4 + b); };
  auto w_full = [&](int s) { return bar0 + 8u * (6 + s); };
  auto w_empty = [&](int s) { return bar0 + 8u * (10 + s); };
  auto d1_full = [&](int b) { return bar0 + 8u * (14 + b); };
  auto d1_empty = [&](int b) { return bar0 + 8u * (18 + b); };
  auto h_full = [&](int b) { return bar0 + 8u * (22 + b); };
  auto h_empty = [&](int b) { return bar0 + 8u * (26 + b); };
  auto d2_full = [&](int b) { return bar0 + 8u * (30 + b); };
  auto d2_empty = [&](int b) { return bar0 + 8u * (32 + b); };
  const uint32_t drain = bar0 + 8u * 34;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_BAR + 384);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + 392);
  float *vec = reinterpret_cast<float *>(smem + off_vec(kb));
  const float *gamma = vec, *beta = vec + p.cp, *s2v = vec + 2 * p.cp, *b2v = vec + 3 * p.cp;
  const float *s1v = vec + 4 * p.cp, *b1v = vec + 4 * p.cp + p.hp;
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;
  const int nh = p.nh;
  const int my_tiles = blockIdx.x < p.total_tiles ? (p.total_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int total = my_tiles * nh;  // hidden chunks this CTA works through
  for (int i = threadIdx.x; i < 2 * p.cp; i += THREADS) vec[i] = p.vec[i];
  for (int i = threadIdx.x; i < 2 * p.cp; i += THREADS) vec[2 * p.cp + i] = p.vec[2 * p.cp + 2 * p.hp + i];
  for (int i = threadIdx.x; i < 2 * p.hp; i += THREADS) vec[4 * p.cp + i] = p.vec[2 * p.cp + i];
  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(a_raw(b), 1);
      mbar_init(a_full(b), 4);
      mbar_init(a_empty(b), 1);
      mbar_init(d2_full(b), 1);
      mbar_init(d2_empty(b), 4);
    }
    for (int b = 0; b < NBUF; ++b) {
      mbar_init(d1_full(b), 1);
      mbar_init(d1_empty(b), 4);
      mbar_init(h_full(b), 4);
      mbar_init(h_empty(b), 1);
    }
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(w_full(s), 1);
      mbar_init(w_empty(s), 1);
    }
    mbar_init(drain, 1);
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
    // ---- TMA producer: the same chunk stream as the MMA issuer ----
    if (lane == 0) {
      tma_prefetch_map(&xmap);
      tma_prefetch_map(&w1map);
      tma_prefetch_map(&w2map);
      int x_issued = 0, ws = 0;
      bool ok = true;
      auto issue_x = [&](int it) -> bool {
        const int b = it & 1;
        if (!mbar_wait(a_empty(b), ((it >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) return false;
        const uint32_t dst = sbase + b * A_BYTES;
        const int row0 = (blockIdx.x + it * gridDim.x) * TILE;
        mbar_arrive_expect_tx(a_raw(b), A_BYTES);
        for (int k = 0; k < kb; ++k) tma_load_3d(dst + k * 16384, &xmap, a_raw(b), k * 64, row0, 0);
        ++x_issued;
        return true;
      };
      auto issue_w = [&](bool first, int h) -> bool {
        const int s = ws % STAGES;
        if (!mbar_wait(w_empty(s), ((ws / STAGES) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) return false;
        const uint32_t dst = sbase + OFF_W + s * W_BYTES;
        mbar_arrive_expect_tx(w_full(s), W_BYTES);
        if (first)
          tma_load_3d(dst, &w1map, w_full(s), 0, h * HC, 0);
        else
          tma_load_3d(dst, &w2map, w_full(s), 0, 0, h * 2);
        ++ws;
        return true;
      };
      if (my_tiles > 0) ok = issue_x(0);
      const int early = nh > 1 ? 1 : 0;  // the next tile's x goes out after this step's W1
      ChunkCursor c1, c2;
      c1.start(nh);
      c2.start(nh);
      for (int j = 0; ok && j < total + LAG; ++j) {
        if (j < total) {
          ok = issue_w(true, c1.chunk);
          if (ok && c1.h == early && c1.it + 1 < my_tiles) ok = issue_x(c1.it + 1);
          c1.advance();
        }
        if (ok && j >= LAG) {
          ok = issue_w(false, c2.chunk);
          c2.advance();
        }
      }
      // Every load issued lands before the CTA exits (immediate unless a consumer gave up).
      for (int i = std::max(0, ws - STAGES); i < ws; ++i) mbar_wait_drain(w_full(i % STAGES), (i / STAGES) & 1, p.err);
      for (int i = std::max(0, x_issued - 2); i < x_issued; ++i) mbar_wait_drain(a_raw(i & 1), (i >> 1) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    const uint32_t idesc1 = idesc_f16_f32(TILE, HC);
    const uint32_t idesc2 = idesc_f16_f32(TILE, p.cp);
    // Base descriptors; every operand below is one of these plus a constant.
    const uint64_t a_desc = sdesc_k_sw128(sbase), w_desc = sdesc_k_sw128(sbase + OFF_W);
    int ws = 0;
    int it1 = 0, h1 = 0, it2 = 0, h2 = 0;  // tile and step of the next first / second GEMM
    for (int j = 0; j < total + LAG; ++j) {
      if (j < total) {  // first GEMM of step j -> D1[j % NBUF]
        const int buf = it1 & 1, db = j % NBUF, s = ws % STAGES;
        if ((h1 == 0 && !warp_wait(a_full(buf), (it1 >> 1) & 1, abort_flag, p.err, kErrWaitMma)) ||
            !warp_wait(d1_empty(db), ((j / NBUF) & 1) ^ 1, abort_flag, p.err, kErrWaitMma) ||
            !warp_wait(w_full(s), (ws / STAGES) & 1, abort_flag, p.err, kErrWaitMma))
          break;
        tc_fence_after();
        const uint64_t ad = desc_add(a_desc, buf * A_BYTES), wd = desc_add(w_desc, s * W_BYTES);
        const uint32_t d = tmem + db * HC;
        umma_first(d, ad, wd, idesc1);
#pragma unroll
        for (int ks = 1; ks < 4 * KB; ++ks)
          umma_acc(d, desc_add(ad, (ks >> 2) * 16384 + (ks & 3) * 32), desc_add(wd, (ks >> 2) * 16384 + (ks & 3) * 32),
                      idesc1);
        umma_commit(w_empty(s));
        umma_commit(d1_full(db));
        if (h1 == nh - 1) umma_commit(a_empty(buf));
        ++ws;
        if (++h1 == nh) {
          h1 = 0;
          ++it1;
        }
      }
      if (j >= LAG) {  // second GEMM of step i = j - LAG: D2[tile] += H[i % NBUF] W2[chunk], H in TMEM
        const int i = j - LAG, buf = it2 & 1, hb = i % NBUF, s = ws % STAGES;
        if (!warp_wait(h_full(hb), (i / NBUF) & 1, abort_flag, p.err, kErrWaitMma) ||
            !warp_wait(w_full(s), (ws / STAGES) & 1, abort_flag, p.err, kErrWaitMma) ||
            (h2 == 0 && !warp_wait(d2_empty(buf), ((it2 >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitMma)))
          break;
        tc_fence_after();
        // H of step i: 128 rows x 128 hidden f16 = 64 TMEM columns at D1[hb]; a K step of
        // 16 hidden channels is 8 columns
        const uint32_t hd = tmem + hb * HC;
        const uint64_t wd = desc_add(w_desc, s * W_BYTES);
        const uint32_t d = tmem + 256 + buf * 128;
        if (h2 == 0)
          umma_ts_first(d, hd, wd, idesc2);
        else
          umma_ts_acc(d, hd, wd, idesc2);
#pragma unroll
        for (int ks = 1; ks < 8; ++ks)
          umma_ts_acc(d, hd + ks * 8, desc_add(wd, (ks >> 2) * W2_KSTRIDE + (ks & 3) * 32), idesc2);
        umma_commit(w_empty(s));
        umma_commit(h_empty(hb));
        if (h2 == nh - 1) umma_commit(d2_full(buf));
        ++ws;
        if (++h2 == nh) {
          h2 = 0;
          ++it2;
        }
      }
    }
    // Every MMA has completed before TMEM is freed, whether or not a consumer gave up.
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else if (warp < 10) {
    // ---- row warps: 2-5 the second epilogue of every tile, 6-9 the LayerNorm of every
    //      x tile (running ahead of the first GEMMs by the two x buffers) ----
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const int row = q * 32 + lane;
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const float inv_c = 1.f / static_cast<float>(p.c);
    bool store_pending = false;
    auto layer_norm = [&](int it) -> bool {  // x tile in place, one thread per row
      const int buf = it & 1;
      if (!warp_wait(a_raw(buf), (it >> 1) & 1, abort_flag, p.err, kErrWaitNormalizer)) return false;
      if (p.normalize) {
        ln_row<XT>(smem + buf * A_BYTES, kb, row, p.c, inv_c, p.eps, gamma, beta);
        fence_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(a_full(buf));
      return true;
    };
    auto second_epilogue = [&](int it) -> bool {  // D2 -> scale2 * acc + b2, 64 channels at a time
      const int buf = it & 1, t = blockIdx.x + it * gridDim.x;
      if (!warp_wait(d2_full(buf), (it >> 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) return false;
      tc_fence_after();
      const int64_t grow = static_cast<int64_t>(t) * TILE + row;
      for (int half = 0; half < kb; ++half) {
        const int col0 = half * 64;
        uint32_t v[2][32];
        const uint32_t d2 = lane_base + 256 + buf * 128 + col0;
        tmem_ld32(d2, v[0]);
        tmem_ld32(d2 + 32, v[1]);
        tmem_ld_wait();
        if (half == kb - 1) {  // the whole accumulator is in registers: release it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(d2_empty(buf));
        }
        const float *sc = s2v + col0, *bi = b2v + col0;
        if (p.out_mode <= kOutTmaAdd) {
          if (lane == 0 && store_pending) bulk_wait_read_all();  // this warp's last store has read the stage
          __syncwarp();
          uint8_t *stage = smem + OFF_O;
#pragma unroll
          for (int j = 0; j < 8; ++j) {  // 8 output channels = one 16-byte chunk of the staged row
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int c = j * 8 + 2 * i;
              const float2 s = *reinterpret_cast<const float2 *>(sc + c);
              const float2 b = *reinterpret_cast<const float2 *>(bi + c);
              const float2 y = f2fma(
                  make_float2(__uint_as_float(v[c >> 5][c & 31]), __uint_as_float(v[c >> 5][(c + 1) & 31])), s, b);
              pk[i] = pack2<OT>(y.x, y.y);
            }
            *reinterpret_cast<uint4 *>(stage + sw128_offset(row, j)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            const uint32_t src = sbase + OFF_O + q * 4096;
            if (p.out_mode == kOutTmaAdd)
              tma_reduce_add_3d(&omap, src, col0, t * TILE + q * 32, 0);
            else
              tma_store_3d(&omap, src, col0, t * TILE + q * 32, 0);
            bulk_commit();
            store_pending = true;
          }
        } else if (grow < p.rows) {
          OT *orow = static_cast<OT *>(p.out) + grow * p.c;
          const bool add = p.out_mode == kOutDirectAdd;
#pragma unroll
          for (int i = 0; i < 64; ++i) {
            const int ch = col0 + i;
            if (ch < p.c) {
              const float y = fmaf(__uint_as_float(v[i >> 5][i & 31]), sc[i], bi[i]);
              orow[ch] = from_f32<OT>(add ? to_f32<OT>(orow[ch]) + y : y);
            }
          }
        }
      }
      return true;
    };
    if (warp >= 6 && KB == 2) {
      // two 64-channel blocks: four threads per row, 32 rows per pass, gamma and beta of the
      // thread's 32 channels held in registers for the whole launch
      const int quarter = lane >> 3, rl = (warp - 6) * 8 + (lane & 7);
      float2 gq[16], bq[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        gq[i] = *reinterpret_cast<const float2 *>(gamma + quarter * 32 + 2 * i);
        bq[i] = *reinterpret_cast<const float2 *>(beta + quarter * 32 + 2 * i);
      }
      for (int it = 0; it < my_tiles; ++it) {
        const int buf = it & 1;
        if (!warp_wait(a_raw(buf), (it >> 1) & 1, abort_flag, p.err, kErrWaitNormalizer)) break;
        if (p.normalize) {
#pragma unroll 1
          for (int pass = 0; pass < TILE / 32; ++pass)
            ln_row_quad<XT>(smem + buf * A_BYTES, pass * 32 + rl, quarter, p.c, inv_c, p.eps, gq, bq);
          fence_async_smem();
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(a_full(buf));
      }
    } else if (warp >= 6) {
      for (int it = 0; it < my_tiles; ++it)
        if (!layer_norm(it)) break;
    } else {
      for (int it = 0; it < my_tiles; ++it)
        if (!second_epilogue(it)) break;
    }
    if (lane == 0 && store_pending) bulk_wait_all();
  } else {
    // ---- first epilogue, four warps taking every chunk:
    //      D1 chunk -> relu(scale1 * acc + b1) -> f16 H, written back over the
    //      first 64 columns of the same accumulator (each half after this
    //      thread has loaded the columns it overwrites) ----
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(q * 32) << 16);
    ChunkCursor cur;
    cur.start(nh);
    for (int j = 0; j < total; ++j, cur.advance()) {
      const int db = j % NBUF, h = cur.chunk;
      const uint32_t ph = (j / NBUF) & 1;
      if (!warp_wait(d1_full(db), ph, abort_flag, p.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      if (!warp_wait(h_empty(db), ph ^ 1, abort_flag, p.err, kErrWaitEpilogue)) break;
      // Each thread converts rows rq, rq + 8 of each 16-lane group of the quarter and the column
      // pairs 8k + 2 cp (the 16x256b TMEM shape), so it needs the scale and bias of 16 of a
      // half's 64 channels, loaded once for its four rows (four different addresses per warp).
      const int rq_cp = lane & 3;
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {  // 64 hidden channels: 64 f32 columns in, 32 packed f16 columns out
        float2 sv[8], bv[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const int c = h * HC + half * 64 + 8 * k + 2 * rq_cp;
          sv[k] = *reinterpret_cast<const float2 *>(s1v + c);
          bv[k] = *reinterpret_cast<const float2 *>(b1v + c);
        }
#pragma unroll
        for (int g = 0; g < 2; ++g) {  // lanes 32 q + 16 g .. 32 q + 16 g + 15
          const uint32_t gbase = lane_base + (static_cast<uint32_t>(16 * g) << 16) + db * HC;
          uint32_t v[32];
          tmem_ld_16x256b_x8(gbase + half * 64, v);
          tmem_ld_wait();
          uint32_t pk[16];
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const float2 y0 = f2fma(make_float2(__uint_as_float(v[4 * k]), __uint_as_float(v[4 * k + 1])), sv[k], bv[k]);
            const float2 y1 =
                f2fma(make_float2(__uint_as_float(v[4 * k + 2]), __uint_as_float(v[4 * k + 3])), sv[k], bv[k]);
            pk[2 * k] = pack_half2_relu(y0.x, y0.y);
            pk[2 * k + 1] = pack_half2_relu(y1.x, y1.y);
          }
          tmem_st_16x128b_x8(gbase + half * 32, pk);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(h_full(db));
        mbar_arrive(d1_empty(db));
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// LayerNorm of [rows][c] (any dtype, any c) into f16 [rows][cp], zero padded:
// the input for the kernel when x cannot go straight into a TMA tile (f32, or
// a row pitch that is not a multiple of 16 bytes).  One warp per row.
template <typename XT>
__global__ void normalize_kernel(const XT *__restrict__ x, int64_t rows, int c, int cp, const float *__restrict__ vec,
                                 float eps, __half *__restrict__ xn) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const XT *xr = x + row * c;
  float v[4];
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ch = lane + 32 * i;
    v[i] = ch < c ? to_f32<XT>(xr[ch]) : 0.f;
    s += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  const float mean = s / static_cast<float>(c);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ch = lane + 32 * i;
    const float d = ch < c ? v[i] - mean : 0.f;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(kFull, q, o);
  const float rstd = rsqrtf(q / static_cast<float>(c) + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ch = lane + 32 * i;
    if (ch < cp) xn[row * cp + ch] = __float2half_rn(ch < c ? (v[i] - mean) * rstd * vec[ch] + vec[cp + ch] : 0.f);
  }
}

// LayerNorm of rows of any width into f16 rows of pitch `pitch` (zero past c),
// for the wide path.  One warp per row, three passes over the row (sum, squared
// deviations, normalised store), the later two served from L1/L2.
template <typename XT>
__global__ void layer_norm_rows_kernel(const XT *__restrict__ x, int64_t rows, int c, int pitch,
                                       const float *__restrict__ gamma, const float *__restrict__ beta, float eps,
                                       __half *__restrict__ xn) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const XT *xr = x + row * c;
  float s = 0.f;
  for (int ch = lane; ch < c; ch += 32) s += to_f32<XT>(xr[ch]);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  const float mean = s / static_cast<float>(c);
  float q = 0.f;
  for (int ch = lane; ch < c; ch += 32) {
    const float d = to_f32<XT>(xr[ch]) - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(kFull, q, o);
  const float rstd = rsqrtf(q / static_cast<float>(c) + eps);
  __half *out = xn + row * pitch;
  for (int ch = lane; ch < pitch; ch += 32)
    out[ch] = __float2half_rn(ch < c ? (to_f32<XT>(xr[ch]) - mean) * rstd * gamma[ch] + beta[ch] : 0.f);
}

// ---------------------------------------------------------------------------
// Weight preparation.
// ---------------------------------------------------------------------------

struct MatrixDev {
  int format, block;
  const void *values, *scales;
};

// f32 value of element i of a matrix of format FMT (exact decode for q8
// block; codes as-is for q8 channel, whose scale is applied in the epilogue).
template <int FMT>
__device__ __forceinline__ float matrix_element(const MatrixDev &m, int64_t i) {
  if (FMT == AF2_WEIGHTS_F32) return static_cast<const float *>(m.values)[i];
  const float code = static_cast<float>(static_cast<const int8_t *>(m.values)[i]);
  if (FMT == AF2_WEIGHTS_Q8_CHANNEL) return code;
  const uint16_t bits = static_cast<const uint16_t *>(m.scales)[i / m.block];
  return code * __half2float(__ushort_as_half(bits));
}

// One block per 32 output columns of one matrix; warp w walks k = w, w + 32,
// ... so each load instruction reads 32 consecutive columns of one row.
// Pass 1 finds the column's scale (the largest magnitude's power of two, or
// the given q8 channel scale), pass 2 writes the f16 operand column.
// Matrix 1 ([c][h]) -> w1p [kb][hp][64]; matrix 2 ([h][c]) -> w2p [hp/64][cp][64].
constexpr int PREP_THREADS = 1024;
constexpr int kPrepBatch = 16;  // values per thread loaded before any is used

// Shared memory of one preparation block: the column maxima and, for pass 2,
// a window of 256 K values of the block's 32 columns, which leaves as whole
// 128-byte operand rows (coalesced) instead of scattered 2-byte stores.
struct PrepShared {
  float red[32][33];
  float col_scale[32];
  __align__(16) __half stage[32][264];
};

template <int FMT>
__device__ __forceinline__ void prep_columns(PrepShared &sh, const MatrixDev &m, bool first, int o, int inner,
                                             int cols, int kpad, int cp, int hp, int c, int h,
                                             const float *__restrict__ b1, const float *__restrict__ b2,
                                             __half *__restrict__ w1p, __half *__restrict__ w2p,
                                             float *__restrict__ vec) {
  float(&red)[32][33] = sh.red;
  float(&col_scale)[32] = sh.col_scale;
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;
  constexpr bool codes = FMT == AF2_WEIGHTS_Q8_CHANNEL;
  // Pass 1: the column's values for this warp (k = warp, warp + 32, ...) in
  // batches, all loads of a batch in flight together.
  // Zero first: a warp whose first k is already past `inner` never enters the
  // loop, and pass 2 writes these registers out as the zero padding.
  float vals[kPrepBatch];
#pragma unroll
  for (int b = 0; b < kPrepBatch; ++b) vals[b] = 0.f;
  float mx = 0.f;
  for (int k0 = warp; k0 < inner; k0 += 32 * kPrepBatch) {
#pragma unroll
    for (int b = 0; b < kPrepBatch; ++b) {
      const int k = k0 + 32 * b;
      vals[b] = (o < cols && k < inner) ? matrix_element<FMT>(m, static_cast<int64_t>(k) * cols + o) : 0.f;
    }
#pragma unroll
    for (int b = 0; b < kPrepBatch; ++b) mx = fmaxf(mx, fabsf(vals[b]));
  }
  red[warp][lane] = mx;
  __syncthreads();
  if (warp == 0) {
    float v = 0.f;
    for (int w = 0; w < 32; ++w) v = fmaxf(v, red[w][lane]);
    float scale = 1.f;
    if (o < cols) {
      if (codes) {
        scale = static_cast<const float *>(m.scales)[o];
      } else if (v > 0.f && isfinite(v)) {
        int e;
        frexpf(v, &e);  // v = f 2^e, f in [0.5, 1)
        scale = ldexpf(1.f, e);
      }
    }
    col_scale[lane] = scale;
    if (first) {
      vec[2 * cp + o] = scale;
      vec[2 * cp + hp + o] = o < h ? b1[o] : 0.f;
    } else {
      vec[2 * cp + 2 * hp + o] = scale;
      vec[3 * cp + 2 * hp + o] = o < c ? b2[o] : 0.f;
    }
  }
  __syncthreads();
  // Pass 2: the f16 operand columns (value / scale, a power of two: exact),
  // staged 256 K values at a time and written as whole operand rows.
  const float inv = codes ? 1.f : 1.f / col_scale[lane];
  const int o0 = o - lane;
  __half *dst_base = first ? w1p : w2p;
  const int rows_per_block = first ? hp : cp;  // operand rows in one 64-wide K block
  for (int k0 = 0; k0 < kpad; k0 += 256) {
    const int kend = min(k0 + 256, kpad);
    if (inner <= 32 * kPrepBatch) {  // the common case: every value is still in registers
#pragma unroll
      for (int b = 0; b < kPrepBatch; ++b) {
        const int k = warp + 32 * b;
        if (k >= k0 && k < kend) sh.stage[lane][k - k0] = __float2half_rn(vals[b] * inv);
      }
      for (int k = k0 + warp; k < kend; k += 32)
        if (k >= 32 * kPrepBatch) sh.stage[lane][k - k0] = __float2half_rn(0.f);
    } else {
      for (int k = k0 + warp; k < kend; k += 32) {
        float w = 0.f;
        if (o < cols && k < inner) w = matrix_element<FMT>(m, static_cast<int64_t>(k) * cols + o) * inv;
        sh.stage[lane][k - k0] = __float2half_rn(w);
      }
    }
    __syncthreads();
    const int blocks = (kend - k0) >> 6;  // 64-wide K blocks in the window: 32 rows x 128 B each
    for (int i = threadIdx.x; i < blocks * 256; i += PREP_THREADS) {
      const int blk = i >> 8, r = (i >> 3) & 31, c16 = i & 7;
      const uint4 v = *reinterpret_cast<const uint4 *>(&sh.stage[r][blk * 64 + c16 * 8]);
      const int64_t kb_index = (k0 >> 6) + blk;
      *reinterpret_cast<uint4 *>(dst_base + (kb_index * rows_per_block + o0 + r) * 64 + c16 * 8) = v;
    }
    __syncthreads();
  }
}

// One block per 32 output columns of one matrix.  Matrix 1 ([c][h]) ->
// w1p [kb][hp][64]; matrix 2 ([h][c]) -> w2p [hp/64][cp][64]; plus the vectors
// gamma beta [cp], scale1 bias1 [hp], scale2 bias2 [cp] (zero padded).
__global__ void __launch_bounds__(PREP_THREADS)
    prep_kernel(MatrixDev m1, MatrixDev m2, const float *__restrict__ gamma, const float *__restrict__ beta,
                const float *__restrict__ b1, const float *__restrict__ b2, int c, int h, int cp, int hp,
                __half *__restrict__ w1p, __half *__restrict__ w2p, float *__restrict__ vec) {
  const int groups1 = hp / 32;
  const bool first = static_cast<int>(blockIdx.x) < groups1;
  const int o = (first ? blockIdx.x : blockIdx.x - groups1) * 32 + (threadIdx.x & 31);
  const MatrixDev &m = first ? m1 : m2;
  const int inner = first ? c : h, cols = first ? h : c, kpad = first ? cp : hp;
  if (blockIdx.x == 0)
    for (int i = threadIdx.x; i < cp; i += PREP_THREADS) {
      vec[i] = i < c ? gamma[i] : 0.f;
      vec[cp + i] = i < c ? beta[i] : 0.f;
    }
  __shared__ PrepShared sh;
  if (m.format == AF2_WEIGHTS_Q8_CHANNEL)
    prep_columns<AF2_WEIGHTS_Q8_CHANNEL>(sh, m, first, o, inner, cols, kpad, cp, hp, c, h, b1, b2, w1p, w2p, vec);
  else if (m.format == AF2_WEIGHTS_Q8_BLOCK)
    prep_columns<AF2_WEIGHTS_Q8_BLOCK>(sh, m, first, o, inner, cols, kpad, cp, hp, c, h, b1, b2, w1p, w2p, vec);
  else
    prep_columns<AF2_WEIGHTS_F32>(sh, m, first, o, inner, cols, kpad, cp, hp, c, h, b1, b2, w1p, w2p, vec);
}

// Bit-exact q8 decode (dtype.ts:86-97; per-channel: the f32 product).
__global__ void dequant_kernel(MatrixDev m, int64_t count, int64_t cols, float *__restrict__ out) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float code = static_cast<float>(static_cast<const int8_t *>(m.values)[i]);
    if (m.format == AF2_WEIGHTS_Q8_CHANNEL)
      out[i] = __fmul_rn(code, static_cast<const float *>(m.scales)[i % cols]);
    else
      out[i] = __fmul_rn(code, __half2float(__ushort_as_half(static_cast<const uint16_t *>(m.scales)[i / m.block])));
  }
}

}  // namespace trn

namespace {

using namespace trn;

MatrixDev to_dev(const af2_matrix &m) { return MatrixDev{m.format, m.block, m.values, m.scales}; }

uint32_t smem_bytes(int kb, int hp) { return off_vec(kb) + (4u * kb * 64 + 2u * hp) * 4u + 1024u; }

template <typename XT, typename OT>
af2_status launch_kernel(af2_ctx *ctx, const CUtensorMap &xmap, const CUtensorMap &w1map, const CUtensorMap &w2map,
                         const CUtensorMap &omap, const Args &a, cudaStream_t stream) {
  auto kernel = a.kb == 2 ? transition_kernel<XT, OT, 2> : transition_kernel<XT, OT, 1>;
  const uint32_t smem = smem_bytes(a.kb, a.hp);
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "transition kernel attributes");
  const int grid = std::min(a.total_tiles, ctx->sm_count);
  LaunchScope scope(ctx, stream, kProfTransition);
  kernel<<<grid, THREADS, smem, stream>>>(xmap, w1map, w2map, omap, a);
  e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "transition kernel launch");
}

template <typename XT>
af2_status launch_out(af2_ctx *ctx, int out_dtype, const CUtensorMap &xmap, const CUtensorMap &w1map,
                      const CUtensorMap &w2map, const CUtensorMap &omap, const Args &a, cudaStream_t stream) {
  if (out_dtype == AF2_F16) return launch_kernel<XT, __half>(ctx, xmap, w1map, w2map, omap, a, stream);
  if (out_dtype == AF2_BF16) return launch_kernel<XT, __nv_bfloat16>(ctx, xmap, w1map, w2map, omap, a, stream);
  return launch_kernel<XT, float>(ctx, xmap, w1map, w2map, omap, a, stream);
}

CUtensorMapDataType map_dtype(int dtype) {
  return dtype == AF2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                           : (dtype == AF2_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32);
}

}  // namespace

TransitionLayout transition_layout(int64_t rows, int64_t c, int64_t h, int x_dtype) {
  TransitionLayout L;
  L.rows = rows;
  L.c = c;
  L.h = h;
  if (c > 128 || h > 1024 || tuning_override("AF2_TRANSITION_WIDE", 0) == 1) {
    // the fused kernel holds C <= 128 channels and H <= 1024 hidden; wider transitions
    // (the MSA transition: 256 -> 1024 -> 256) take the two-GEMM path, which
    // AF2_TRANSITION_WIDE=1 also selects for shapes the fused kernel holds
    L.wide = true;
    L.k1 = align_up(c, 64);
    L.n1 = linear_cols_pad(h);
    L.k2 = align_up(h, 64);
    L.n2 = linear_cols_pad(c);
    L.hid_pitch = align_up(h, 8);
    const int64_t cap = std::max<int64_t>(128, ((int64_t)256 << 20) / (L.hid_pitch * 2) / 128 * 128);
    L.chunk_rows = std::min(rows, cap);
    size_t off = 0;
    auto take = [&](size_t bytes) {
      const size_t at = off;
      off = align_up(off + bytes, 256);
      return at;
    };
    L.off_w1 = take((size_t)L.k1 * L.n1 * 2);
    L.off_s1 = take((size_t)L.n1 * 4);
    L.off_b1 = take((size_t)L.n1 * 4);
    L.off_w2 = take((size_t)L.k2 * L.n2 * 2);
    L.off_s2 = take((size_t)L.n2 * 4);
    L.off_b2 = take((size_t)L.n2 * 4);
    L.off_xn = take((size_t)L.chunk_rows * L.k1 * 2);
    L.off_hid = take((size_t)L.chunk_rows * L.hid_pitch * 2);
    L.total = off;
    return L;
  }
  L.cp = c <= 64 ? 64 : 128;
  L.hp = (h + 127) / 128 * 128;
  L.fast_in = x_dtype != AF2_F32 && c % 8 == 0;
  L.chunk_rows = L.fast_in ? rows : std::min<int64_t>(rows, 65536);
  size_t off = 0;
  L.off_w1 = off;
  off = align_up(off + (size_t)L.cp * L.hp * 2, 256);
  L.off_w2 = off;
  off = align_up(off + (size_t)L.cp * L.hp * 2, 256);
  L.off_vec = off;
  off = align_up(off + (size_t)(4 * L.cp + 2 * L.hp) * 4, 256);
  L.off_xn = off;
  if (!L.fast_in) off = align_up(off + (size_t)L.chunk_rows * L.cp * 2, 256);
  L.total = off;
  return L;
}

// The key of a transition's prepared weights in the context's weight cache.
static WeightKey transition_key(const TransitionLayout &L, const af2_transition_weights &w) {
  WeightKey key;
  key.kind = kWeightsTransition;
  const void *ptrs[8] = {w.layer_norm_scale, w.layer_norm_offset, w.first_weight.values, w.first_weight.scales,
                         w.first_bias,       w.second_weight.values, w.second_weight.scales, w.second_bias};
  for (int i = 0; i < 8; ++i) key.ptr[i] = ptrs[i];
  const int64_t dims[6] = {L.c, L.h, w.first_weight.format * 65536 + w.first_weight.block,
                           w.second_weight.format * 65536 + w.second_weight.block, L.wide ? 1 : 0, L.cp};
  for (int i = 0; i < 6; ++i) key.dim[i] = dims[i];
  return key;
}

af2_status transition_prepare(af2_ctx *ctx, const TransitionLayout &L, const af2_transition_weights &w,
                              void *workspace, cudaStream_t stream) {
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const unsigned blocks = static_cast<unsigned>(L.hp / 32 + L.cp / 32);
  LaunchScope scope(ctx, stream, kProfTransitionPrepare);
  prep_kernel<<<blocks, PREP_THREADS, 0, stream>>>(
      to_dev(w.first_weight), to_dev(w.second_weight), w.layer_norm_scale, w.layer_norm_offset, w.first_bias,
      w.second_bias, (int)L.c, (int)L.h, (int)L.cp, (int)L.hp, reinterpret_cast<__half *>(ws + L.off_w1),
      reinterpret_cast<__half *>(ws + L.off_w2), reinterpret_cast<float *>(ws + L.off_vec));
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "transition weight preparation");
}

// The wide path, per row chunk: LayerNorm -> f16 copy; hidden = relu(xn W1 + b1) (f16, HBM);
// out (=, +=) hidden W2 + b2 -- the reference's own kernel sequence (transition.ts:264-361),
// with both GEMMs on the shared tcgen05 linear kernel.
static af2_status transition_launch_wide(af2_ctx *ctx, const TransitionLayout &L, const void *x, int x_dtype,
                                         const af2_transition_weights &w, double eps, int residual, void *out,
                                         int out_dtype, void *workspace, cudaStream_t stream) {
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  // the prepared weights: the layout's prefix [0, off_xn), in the weight cache or the workspace
  PreparedRegion pw;
  af2_status st = prepared_region(ctx, transition_key(L, w), L.off_xn, ws, true, &pw);
  if (st != AF2_OK) return st;
  uint8_t *wp = pw.base;
  float *s1 = reinterpret_cast<float *>(wp + L.off_s1), *b1 = reinterpret_cast<float *>(wp + L.off_b1);
  float *s2 = reinterpret_cast<float *>(wp + L.off_s2), *b2 = reinterpret_cast<float *>(wp + L.off_b2);
  if (pw.fresh) {
    PrepJob jobs[2];
    jobs[0] = PrepJob{w.first_weight, L.c, L.h, L.k1, L.n1, 1.f, wp + L.off_w1, s1};
    jobs[1] = PrepJob{w.second_weight, L.h, L.c, L.k2, L.n2, 1.f, wp + L.off_w2, s2};
    VectorSegments v{};
    v.add(w.first_bias, L.h, L.n1, b1);
    v.add(w.second_bias, L.c, L.n2, b2);
    if ((st = prepare_matrices(ctx, jobs, 2, stream)) != AF2_OK || (st = pad_vectors(ctx, v, stream)) != AF2_OK)
      return st;
  }
  const size_t xb = x_dtype == AF2_F32 ? 4 : 2, ob = out_dtype == AF2_F32 ? 4 : 2;
  __half *xn = reinterpret_cast<__half *>(ws + L.off_xn), *hid = reinterpret_cast<__half *>(ws + L.off_hid);
  for (int64_t r0 = 0; r0 < L.rows; r0 += L.chunk_rows) {
    const int64_t rows = std::min(L.chunk_rows, L.rows - r0);
    const void *xsrc = static_cast<const uint8_t *>(x) + r0 * L.c * xb;
    {
      const int warps = 8;
      const unsigned blocks = (unsigned)((rows + warps - 1) / warps);
      LaunchScope scope(ctx, stream, kProfTransitionNormalize);
      const int c = (int)L.c, pitch = (int)L.k1;
      const float e = static_cast<float>(eps);
      if (x_dtype == AF2_F32)
        layer_norm_rows_kernel<float><<<blocks, warps * 32, 0, stream>>>(
            static_cast<const float *>(xsrc), rows, c, pitch, w.layer_norm_scale, w.layer_norm_offset, e, xn);
      else if (x_dtype == AF2_F16)
        layer_norm_rows_kernel<__half><<<blocks, warps * 32, 0, stream>>>(
            static_cast<const __half *>(xsrc), rows, c, pitch, w.layer_norm_scale, w.layer_norm_offset, e, xn);
      else
        layer_norm_rows_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, stream>>>(
            static_cast<const __nv_bfloat16 *>(xsrc), rows, c, pitch, w.layer_norm_scale, w.layer_norm_offset, e,
            xn);
      const cudaError_t err = cudaGetLastError();
      if (err != cudaSuccess) return cuda_fail(ctx, err, "transition normalisation");
    }
    LinearOperands g1;
    g1.a = xn;
    g1.lda = L.k1;
    g1.w = wp + L.off_w1;
    g1.scale = s1;
    g1.bias = b1;
    g1.rows = rows;
    g1.inner = L.c;
    g1.cols = L.h;
    g1.out = hid;
    g1.ldo = L.hid_pitch;
    g1.out_dtype = AF2_F16;
    g1.relu = 1;
    g1.prof = kProfTransitionLinear;
    if ((st = linear_launch(ctx, g1, stream)) != AF2_OK) return st;
    LinearOperands g2;
    g2.a = hid;
    g2.lda = L.hid_pitch;
    g2.w = wp + L.off_w2;
    g2.scale = s2;
    g2.bias = b2;
    g2.rows = rows;
    g2.inner = L.h;
    g2.cols = L.c;
    g2.out = static_cast<uint8_t *>(out) + r0 * L.c * ob;
    g2.ldo = L.c;
    g2.out_dtype = out_dtype;
    g2.residual = residual;
    g2.prof = kProfTransitionLinear;
    if ((st = linear_launch(ctx, g2, stream)) != AF2_OK) return st;
  }
  return AF2_OK;
}

af2_status transition_launch(af2_ctx *ctx, const TransitionLayout &L, const void *x, int x_dtype,
                             const af2_transition_weights &w, double eps, int residual, void *out, int out_dtype,
                             void *workspace, cudaStream_t stream) {
  if (L.wide) return transition_launch_wide(ctx, L, x, x_dtype, w, eps, residual, out, out_dtype, workspace, stream);
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  // the prepared weights: the layout's prefix [0, off_xn), in the weight cache or the workspace
  PreparedRegion pw;
  af2_status st = prepared_region(ctx, transition_key(L, w), L.off_xn, ws, true, &pw);
  if (st != AF2_OK) return st;
  uint8_t *wp = pw.base;
  if (pw.fresh && (st = transition_prepare(ctx, L, w, wp, stream)) != AF2_OK) return st;
  const int kb = static_cast<int>(L.cp / 64);
  CUtensorMap w1map, w2map;
  if (!encode_map_3d(&w1map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wp + L.off_w1, 64, L.hp, kb, 128,
                     (uint64_t)L.hp * 128, 64, HC, kb, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&w2map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wp + L.off_w2, 64, L.cp, L.hp / 64, 128,
                     (uint64_t)L.cp * 128, 64, L.cp, 2, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the transition weights");
  const size_t xb = x_dtype == AF2_F32 ? 4 : 2, ob = out_dtype == AF2_F32 ? 4 : 2;
  const bool tma_out = out_dtype != AF2_F32 && L.c % 8 == 0;
  Args a{};
  a.vec = reinterpret_cast<const float *>(wp + L.off_vec);
  a.c = (int)L.c;
  a.cp = (int)L.cp;
  a.kb = kb;
  a.hp = (int)L.hp;
  a.nh = (int)(L.hp / HC);
  a.eps = static_cast<float>(eps);
  a.err = ctx->err_word;
  a.out_mode = tma_out ? (residual ? kOutTmaAdd : kOutTmaStore) : (residual ? kOutDirectAdd : kOutDirect);
  for (int64_t r0 = 0; r0 < L.rows; r0 += L.chunk_rows) {
    const int64_t rows = std::min(L.chunk_rows, L.rows - r0);
    const void *xsrc = static_cast<const uint8_t *>(x) + r0 * L.c * xb;
    void *odst = static_cast<uint8_t *>(out) + r0 * L.c * ob;
    CUtensorMap xmap, omap;
    int xdt = x_dtype;
    if (!L.fast_in) {
      __half *xn = reinterpret_cast<__half *>(ws + L.off_xn);
      const int warps = 8;
      const unsigned blocks = (unsigned)((rows + warps - 1) / warps);
      {
        LaunchScope scope(ctx, stream, kProfTransitionNormalize);
        const float *vec = reinterpret_cast<const float *>(wp + L.off_vec);
        if (x_dtype == AF2_F32)
          normalize_kernel<float><<<blocks, warps * 32, 0, stream>>>(static_cast<const float *>(xsrc), rows, a.c,
                                                                     a.cp, vec, a.eps, xn);
        else if (x_dtype == AF2_F16)
          normalize_kernel<__half><<<blocks, warps * 32, 0, stream>>>(static_cast<const __half *>(xsrc), rows, a.c,
                                                                      a.cp, vec, a.eps, xn);
        else
          normalize_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, stream>>>(
              static_cast<const __nv_bfloat16 *>(xsrc), rows, a.c, a.cp, vec, a.eps, xn);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return cuda_fail(ctx, e, "transition normalisation");
      }
      xsrc = xn;
      xdt = AF2_F16;
      if (!encode_map_3d(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, xsrc, L.cp, rows, 1, L.cp * 2,
                         (uint64_t)rows * L.cp * 2, 64, TILE, 1, CU_TENSOR_MAP_SWIZZLE_128B))
        return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the normalised activations");
    } else if (!encode_map_3d(&xmap, map_dtype(x_dtype), xsrc, L.c, rows, 1, L.c * xb, (uint64_t)rows * L.c * xb,
                              64, TILE, 1, CU_TENSOR_MAP_SWIZZLE_128B)) {
      return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the activations");
    }
    if (tma_out) {
      if (!encode_map_3d(&omap, map_dtype(out_dtype), odst, L.c, rows, 1, L.c * ob, (uint64_t)rows * L.c * ob, 64,
                         32, 1, CU_TENSOR_MAP_SWIZZLE_128B))
        return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the output");
    } else {
      omap = xmap;  // unused by the direct-store modes
    }
    a.out = odst;
    a.rows = rows;
    a.total_tiles = (int)((rows + TILE - 1) / TILE);
    a.normalize = L.fast_in ? 1 : 0;
    if (xdt == AF2_BF16)
      st = launch_out<__nv_bfloat16>(ctx, out_dtype, xmap, w1map, w2map, omap, a, stream);
    else
      st = launch_out<__half>(ctx, out_dtype, xmap, w1map, w2map, omap, a, stream);
    if (st != AF2_OK) return st;
  }
  return AF2_OK;
}

af2_status dequant_launch(af2_ctx *ctx, const af2_matrix &m, int64_t inner, int64_t cols, float *out,
                          cudaStream_t stream) {
  const int64_t count = inner * cols;
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((count + threads - 1) / threads, 4LL * ctx->sm_count * 8);
  LaunchScope scope(ctx, stream, kProfDequant);
  dequant_kernel<<<std::max(1u, blocks), threads, 0, stream>>>(to_dev(m), count, cols, out);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "q8 decode");
}

}  // namespace af2
