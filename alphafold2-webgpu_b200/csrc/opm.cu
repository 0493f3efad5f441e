// opm.cu -- the outer-product mean on sm_100a.
//
// Reference: src/evoformer/outer-product-mean.ts:114-153 (LayerNorm over c_m),
// :189-231 (left/right = mask * (LN(m) W + b), one GEMM with 2c columns),
// :317-332 (pair counts), :350-417 (outer[i,j,a,b] = sum_s left[s,i,a]
// right[s,j,b]), :433-486 (out = (outer W_o + b_o) / (eps + count)) and
// :506-536 (residue blocks bounding the outer scratch); the in-model encoder
// is src/evoformer/block.ts:1115-1246.  The reference's own CPU formulation is
// test/outer-product-mean-reference.gpu.test.ts:22-79.
//
// Launches per call (weights prepared first):
//   lnproj     (16-bit MSA, fused layouts) LayerNorm and projection in one
//              kernel, in place of normalize + project below
//   normalize  LayerNorm of every MSA row -> f16 [S*N][c_m]
//   project    the shared tcgen05 GEMM: LN(m) [W_left | W_right], bias, times
//              the row's mask, split into left and right, f16 [S][N][c]
//   count      1 / (norm_eps + sum_s mask[s,i] mask[s,j]) per pair
//   fused      (S <= 1024, c_z <= 128) the outer products and the output
//              projection in one kernel, the outer products kept on chip; the
//              normalisation then orders rows residue-major and the
//              projection writes left [c][N][S] and right [N][c][S], so both
//              operands are K-major (sequences contiguous); otherwise,
//   per residue block of output rows i:
//     outer    tcgen05 GEMM over s with both operands read MN-major straight
//              from the [S][N*c] layouts: a 128 x 256 tile is 4 residues i x
//              8 residues j (x 32 x 32 channels); its epilogue writes each pair
//              row (i, j) as 1024 contiguous f16 (index a*c + b, the order of
//              W_o's rows), scaled by 2^-k with 2^k >= S to stay in f16 range
//     output   the shared GEMM: outer W_o (column scales carry the 2^k back),
//              + b_o, times the pair's 1/(eps + count), written or added
// Blocking over residues bounds the outer scratch only: every output element
// is computed the same way whatever the block, so results are bit-identical.
#include <algorithm>
#include <cmath>
#include <string>
#include <type_traits>

#include "af2_device.cuh"
#include "af2_internal.h"

namespace af2 {
namespace opm {

constexpr int C = 32;  // outer channels c: the outer tile maps 32 channels to 32 TMEM lanes / columns

// ---- LayerNorm over c_m (<= 256), one warp per MSA row ----
// VEC: c_m = 256 with 16-byte rows: each lane holds 8 contiguous channels
// (two float4 or one 16-byte load of 16-bit values) and writes them back as one
// 16-byte store of f16.  Otherwise lanes stride the channels one by one.
template <typename MT, bool VEC>
__global__ void norm_kernel(const MT *__restrict__ m, int64_t rows, int cm, int cmp, const float *__restrict__ gamma,
                            const float *__restrict__ beta, float eps, __half *__restrict__ xn, int n_full, int col0,
                            int cols, int seqs, const float *__restrict__ mask_in, float *__restrict__ mask_out,
                            int split, int m_cols, int m_col0) {
  // m holds m_cols residue columns from m_col0 (n_full and col0 for a whole MSA; the rank's own
  // columns, m_col0 = 0, for a row-sharded one); the mask is always the whole [S][n_full]
  // split (f32 precision mode): rows of 3 cmp, [f16(v) | f16(v) | f16(v - f16(v))], the A operand of a
  // projection whose weights are stacked [W_hi; W_lo; W_hi]
  // local row of the residue columns [col0, col0 + cols) of an [S][n_full] MSA:
  // row = s * cols + j, or with seqs > 0 (residue-major order) row = j * seqs + s
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t sq = seqs > 0 ? row % seqs : row / cols, jl = seqs > 0 ? row / seqs : row % cols;
  const int64_t src = sq * n_full + col0 + jl;
  if (lane == 0) mask_out[row] = mask_in[src];
  const MT *xr = m + (sq * m_cols + m_col0 + jl) * cm;
  float v[8];
  if (VEC) {
    if constexpr (sizeof(MT) == 4) {
      const float4 a = reinterpret_cast<const float4 *>(xr)[2 * lane], b = reinterpret_cast<const float4 *>(xr)[2 * lane + 1];
      v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    } else {
      unpack8<MT>(reinterpret_cast<const uint4 *>(xr)[lane], v);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ch = lane + 32 * i;
      v[i] = ch < cm ? to_f32<MT>(xr[ch]) : 0.f;
    }
  }
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) s += v[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(kFull, s, o);
  const float mean = s / static_cast<float>(cm);
  float q = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int ch = VEC ? lane * 8 + i : lane + 32 * i;
    const float d = ch < cm ? v[i] - mean : 0.f;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(kFull, q, o);
  const float rstd = rsqrtf(q / static_cast<float>(cm) + eps);
  if (VEC) {
    const float4 g0 = reinterpret_cast<const float4 *>(gamma)[2 * lane], g1 = reinterpret_cast<const float4 *>(gamma)[2 * lane + 1];
    const float4 b0 = reinterpret_cast<const float4 *>(beta)[2 * lane], b1 = reinterpret_cast<const float4 *>(beta)[2 * lane + 1];
    const float g[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    uint32_t pk[4], lo[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float y0 = (v[2 * i] - mean) * rstd * g[2 * i] + b[2 * i];
      const float y1 = (v[2 * i + 1] - mean) * rstd * g[2 * i + 1] + b[2 * i + 1];
      pk[i] = pack_half2(y0, y1);
      const __half2 h = *reinterpret_cast<const __half2 *>(&pk[i]);
      lo[i] = pack_half2(y0 - __low2float(h), y1 - __high2float(h));
    }
    const int64_t pitch = split ? 3 * cmp : cmp;
    const uint4 hv = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    reinterpret_cast<uint4 *>(xn + row * pitch)[lane] = hv;
    if (split) {
      reinterpret_cast<uint4 *>(xn + row * pitch + cmp)[lane] = hv;
      reinterpret_cast<uint4 *>(xn + row * pitch + 2 * cmp)[lane] = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
  } else {
    const int64_t pitch = split ? 3 * cmp : cmp;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ch = lane + 32 * i;
      if (ch < cmp) {
        const float y = ch < cm ? (v[i] - mean) * rstd * gamma[ch] + beta[ch] : 0.f;
        const __half h = __float2half_rn(y);
        xn[row * pitch + ch] = h;
        if (split) {
          xn[row * pitch + cmp + ch] = h;
          xn[row * pitch + 2 * cmp + ch] = __float2half_rn(y - __half2float(h));
        }
      }
    }
  }
}

// ---- pair counts: rowscale[i*N + j] = 1 / (norm_eps + sum_s mask[s,i] mask[s,j]) ----
// A 64 x 64 block of pairs per CTA of 128 threads, each thread a 4 (i) x 8 (j)
// register block of contiguous pairs fed by 16-byte shared-memory loads (three
// loads per 32 FMAs), 32 MSA rows of both residue ranges at a time; every count
// sums s in order.
constexpr int CNT_TILE = 64, CNT_S = 32, CNT_THREADS = 256;
// 1 / (eps + sum_s mask[s][i] mask[s][j]) for a 64 x 64 block of pairs: 256 threads, each a 4 x 4
// register block summed with packed f32x2 FMAs (two j per instruction), over chunks of 32
// sequences staged in shared memory while the next chunk's loads are in flight.  Every product
// is summed in ascending s, so the result does not depend on the blocking.
__global__ void __launch_bounds__(CNT_THREADS) count_kernel(const float *__restrict__ mask, int s_count, int n,
                                                            int row0, int rows, float norm_eps,
                                                            float *__restrict__ rowscale) {
  // rows i in [row0, row0 + rows), stored from row 0 of rowscale
  __shared__ __align__(16) float mi[CNT_S][CNT_TILE];
  __shared__ __align__(16) float mj[CNT_S][CNT_TILE];
  const int i0 = row0 + blockIdx.y * CNT_TILE, j0 = blockIdx.x * CNT_TILE;
  const int i_end = row0 + rows;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;  // j0 + 4 tx .., i0 + 4 ty ..
  float2 acc[4][2];
#pragma unroll
  for (int u = 0; u < 4; ++u) acc[u][0] = acc[u][1] = make_float2(0.f, 0.f);
  constexpr int kPer = CNT_S * CNT_TILE / CNT_THREADS;
  float ra[kPer], rb[kPer];
  auto fetch = [&](int s0) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int e = threadIdx.x + k * CNT_THREADS, r = e / CNT_TILE, c = e % CNT_TILE;
      const int64_t s = s0 + r;
      const bool sl = s < s_count;
      ra[k] = (sl && i0 + c < i_end) ? mask[s * n + i0 + c] : 0.f;
      rb[k] = (sl && j0 + c < n) ? mask[s * n + j0 + c] : 0.f;
    }
  };
  fetch(0);
  for (int s0 = 0; s0 < s_count; s0 += CNT_S) {
#pragma unroll
    for (int k = 0; k < kPer; ++k) {
      const int e = threadIdx.x + k * CNT_THREADS, r = e / CNT_TILE, c = e % CNT_TILE;
      mi[r][c] = ra[k];
      mj[r][c] = rb[k];
    }
    __syncthreads();
    if (s0 + CNT_S < s_count) fetch(s0 + CNT_S);
#pragma unroll 8
    for (int r = 0; r < CNT_S; ++r) {
      const float4 a = *reinterpret_cast<const float4 *>(&mi[r][ty * 4]);
      const float4 b = *reinterpret_cast<const float4 *>(&mj[r][tx * 4]);
      const float av[4] = {a.x, a.y, a.z, a.w};
      const float2 b01 = make_float2(b.x, b.y), b23 = make_float2(b.z, b.w);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        acc[u][0] = f2fma(f2(av[u]), b01, acc[u][0]);
        acc[u][1] = f2fma(f2(av[u]), b23, acc[u][1]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const int i = i0 + ty * 4 + u;
    if (i >= i_end) continue;
    const float vals[4] = {acc[u][0].x, acc[u][0].y, acc[u][1].x, acc[u][1].y};
#pragma unroll
    for (int v = 0; v < 4; ++v) {
      const int j = j0 + tx * 4 + v;
      if (j < n) rowscale[static_cast<int64_t>(i - row0) * n + j] = 1.f / (norm_eps + vals[v]);
    }
  }
}

// bias[o] += sum_k beta[k] W[k][o] over the projection's 2c columns (left then
// right): the LayerNorm's beta folded into the biases.  One warp per column,
// lanes splitting k, f64 sums.
__global__ void fold_beta_kernel(const float *__restrict__ beta, const float *__restrict__ wl,
                                 const float *__restrict__ wr, int cm, int c, float *__restrict__ bias) {
  const int o = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (o >= 2 * c) return;
  const float *w = o < c ? wl : wr;
  const int col = o < c ? o : o - c;
  double acc = 0.0;
  for (int k = lane; k < cm; k += 32) acc += static_cast<double>(beta[k]) * w[static_cast<int64_t>(k) * c + col];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(kFull, acc, off);
  if (lane == 0) bias[o] += static_cast<float>(acc);
}

// ---- LayerNorm and the left/right projection in one kernel ----
// For a 16-bit MSA and the fused outer-product layouts.  A tile is 128
// sequences s of one residue i: TMA lands m[s][i][:] as 128 K-major rows of
// c_m in 64-channel 128B-swizzled chunks (zero past c_m); eight warps
// normalise it in place to (x - mean) rstd (two threads per row, each over
// alternate chunks, the statistics combined by one shuffle); one tcgen05 GEMM
// per tile gives D[s][0..63] = LN(m) [W_left | W_right], with the LayerNorm's
// gamma folded into the weight rows and beta into the biases; four warps apply
// the column scale, the bias and the mask and write left[a][i][s] and
// right[i][b][s] (the lanes
// of a warp hold consecutive sequences, so each store covers 64 contiguous
// bytes).  The normalised MSA never reaches HBM.
constexpr int LP_THREADS = 448;  // warp 0 TMA, 1 MMA, 2-9 LayerNorm, 10-13 epilogue
constexpr int LP_STAGES = 3;
constexpr uint32_t LP_CHUNK = 128 * 128;            // 128 rows x 64 channels, 16-bit
constexpr uint32_t LP_STAGE = 4 * LP_CHUNK;         // c_m <= 256
constexpr uint32_t LP_W_CHUNK = 64 * 128;           // 64 output columns x 64 channels
constexpr uint32_t LP_OFF_STAGE = 4 * LP_W_CHUNK;   // 32 KB of weights first
constexpr uint32_t LP_OFF_BAR = LP_OFF_STAGE + LP_STAGES * LP_STAGE;
constexpr uint32_t LP_OFF_VEC = LP_OFF_BAR + 256;  // column scales and biases, 64 f32 each
constexpr uint32_t LP_SMEM = LP_OFF_VEC + 512 + 1024;

struct LnProjArgs {
  const float *scale, *bias;  // per output column (64: left then right); gamma and beta are folded in
  const float *mask;          // [S][n_full]
  int m_row0;                 // the MSA map's column of residue row0 (row0 for a whole MSA, 0 for the rank's own)
  const __half *w;            // [chunks][64][64] f16 operand rows
  __half *left, *right;       // left [c][rows][pitch]; right (this rank's block) [rows][c][pitch]
  int64_t n_full, rows, pitch;
  int row0, s_count, cm, chunks, n_sb, total_tiles;
  float eps;
  unsigned int *err;
};

template <typename MT>
__global__ void __launch_bounds__(LP_THREADS, 1)
    lnproj_kernel(const __grid_constant__ CUtensorMap mmap, const LnProjArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + LP_OFF_BAR;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto ready = [&](int s) { return bar0 + 8u * (LP_STAGES + s); };
  auto empty = [&](int s) { return bar0 + 8u * (2 * LP_STAGES + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (3 * LP_STAGES + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (3 * LP_STAGES + 2 + b); };
  const uint32_t drain = bar0 + 8u * (3 * LP_STAGES + 4);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + LP_OFF_BAR + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + LP_OFF_BAR + 200);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;
  const uint32_t stage_bytes = static_cast<uint32_t>(p.chunks) * LP_CHUNK;

  // weights: chunk kc, output column r -> 128B-swizzled K-major rows
  for (int q = threadIdx.x; q < p.chunks * 64 * 8; q += LP_THREADS) {
    const int kc = q >> 9, r = (q >> 3) & 63, c16 = q & 7;
    const uint4 v = *reinterpret_cast<const uint4 *>(p.w + (static_cast<size_t>(kc) * 64 + r) * 64 + c16 * 8);
    *reinterpret_cast<uint4 *>(smem + kc * LP_W_CHUNK + sw128_offset(r, c16)) = v;
  }
  float *vsm = reinterpret_cast<float *>(smem + LP_OFF_VEC);  // [0, 64) scales, [64, 128) biases
  if (threadIdx.x < 128) vsm[threadIdx.x] = threadIdx.x < 64 ? p.scale[threadIdx.x] : p.bias[threadIdx.x - 64];
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < LP_STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(ready(s), 8);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 4);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 128);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_map(&mmap);
      int it = 0;
      for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
        const int s = it % LP_STAGES;
        if (!mbar_wait(empty(s), ((it / LP_STAGES) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) break;
        const int i = t / p.n_sb, sb = t - i * p.n_sb;
        const uint32_t dst = sbase + LP_OFF_STAGE + s * LP_STAGE;
        mbar_arrive_expect_tx(full(s), stage_bytes);
        for (int kc = 0; kc < p.chunks; ++kc)
          tma_load_3d(dst + kc * LP_CHUNK, &mmap, full(s), kc * 64, p.m_row0 + i, sb * 128);
      }
      // every load issued has landed before the CTA exits (immediate unless a consumer gave up)
      for (int j = it > LP_STAGES ? it - LP_STAGES : 0; j < it; ++j)
        mbar_wait_drain(full(j % LP_STAGES), (j / LP_STAGES) & 1, p.err);
    }
  } else if (warp == 1) {
    // the whole warp runs the issue loop; one elected lane issues
    constexpr uint32_t kIdesc = idesc_f16_f32(128, 64);
    const uint64_t w_base = sdesc_k_sw128(sbase), x_base = sdesc_k_sw128(sbase + LP_OFF_STAGE);
    int s = 0, buf = 0;
    uint32_t ph = 0, bph = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x) {
      if (!warp_wait(acc_empty(buf), bph ^ 1, abort_flag, p.err, kErrWaitMma) ||
          !warp_wait(ready(s), ph, abort_flag, p.err, kErrWaitMma))
        break;
      tc_fence_after();
      const uint64_t xd = x_base + s * (LP_STAGE >> 4);
      const uint32_t d = tmem + buf * 64;
      for (int kc = 0; kc < p.chunks; ++kc) {
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          const uint64_t ad = xd + ((kc * LP_CHUNK + ks * 32) >> 4);
          const uint64_t bd = w_base + ((kc * LP_W_CHUNK + ks * 32) >> 4);
          if (kc == 0 && ks == 0)
            umma_first(d, ad, bd, kIdesc);
          else
            umma_acc(d, ad, bd, kIdesc);
        }
      }
      umma_commit(empty(s));
      umma_commit(acc_full(buf));
      if (++s == LP_STAGES) {
        s = 0;
        ph ^= 1;
      }
      buf ^= 1;
      if (buf == 0) bph ^= 1;
    }
    // Every MMA has completed before TMEM is freed, whether or not a consumer gave up.
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else if (warp < 10) {
    // ---- LayerNorm in place: a warp takes 16 rows; lanes l and l + 16 share a row, ----
    // ---- over chunks kc = half, half + 2 (8 lanes of a quarter-warp: 8 rows, no conflicts) ----
    const int row = (warp - 2) * 16 + (lane & 15), half = lane >> 4;
    const float inv_cm = 1.f / static_cast<float>(p.cm);
    const bool ragged = p.cm != p.chunks * 64;
    int it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++it) {
      const int s = it % LP_STAGES;
      if (!warp_wait(full(s), (it / LP_STAGES) & 1, abort_flag, p.err, kErrWaitNormalizer)) break;
      uint8_t *tile = smem + LP_OFF_STAGE + s * LP_STAGE;
      auto piece = [&](int kc, int c16) { return tile + kc * LP_CHUNK + sw128_offset(row, c16); };
      // statistics over values shifted by the row's first channel (both threads use it)
      const float x0 = unpack2<MT>(*reinterpret_cast<const uint32_t *>(piece(0, 0))).x;
      const float2 neg_x0 = f2(-x0);
      float2 s1 = f2(0.f), s2 = f2(0.f);
      for (int kc = half; kc < p.chunks; kc += 2) {
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          const uint4 v = *reinterpret_cast<const uint4 *>(piece(kc, c16));
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            float2 d = f2add(unpack2<MT>(w[e]), neg_x0);
            if (ragged) {  // channels past c_m (zero-filled) stay out of the statistics
              const int ch = kc * 64 + c16 * 8 + 2 * e;
              d.x = ch < p.cm ? d.x : 0.f;
              d.y = ch + 1 < p.cm ? d.y : 0.f;
            }
            s1 = f2add(s1, d);
            s2 = f2fma(d, d, s2);
          }
        }
      }
      float a1 = s1.x + s1.y, a2 = s2.x + s2.y;
      a1 += __shfl_xor_sync(kFull, a1, 16);
      a2 += __shfl_xor_sync(kFull, a2, 16);
      const float m1 = a1 * inv_cm;
      const float mean = x0 + m1;
      const float rstd = rsqrtf(fmaxf(a2 * inv_cm - m1 * m1, 0.f) + p.eps);
      const float2 r2 = f2(rstd), sh2 = f2(-mean * rstd);
      for (int kc = half; kc < p.chunks; kc += 2) {
#pragma unroll
        for (int c16 = 0; c16 < 8; ++c16) {
          uint8_t *ptr = piece(kc, c16);
          const uint4 v = *reinterpret_cast<const uint4 *>(ptr);
          const uint32_t w[4] = {v.x, v.y, v.z, v.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 y = f2fma(unpack2<MT>(w[e]), r2, sh2);
            o[e] = pack_half2(y.x, y.y);
          }
          *reinterpret_cast<uint4 *>(ptr) = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(ready(s));
    }
  } else {
    // ---- epilogue: scale, bias, mask; left[a][i][s], right[i][b][s] ----
    const int q = warp & 3;
    int tile_it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++tile_it) {
      const int buf = tile_it & 1;
      if (!warp_wait(acc_full(buf), (tile_it >> 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const int i = t / p.n_sb, sb = t - i * p.n_sb;
      const int sq = sb * 128 + q * 32 + lane;
      const bool live = sq < p.s_count;
      const float mk = live ? p.mask[static_cast<int64_t>(sq) * p.n_full + p.row0 + i] : 0.f;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * 64;
#pragma unroll
      for (int part = 0; part < 2; ++part) {  // 0: left (columns 0-31), 1: right (32-63)
        uint32_t v[32];
        __syncwarp();
        tmem_ld32(taddr + part * 32, v);
        tmem_ld_wait();
        if (part == 1) {  // the accumulator is free once every lane has read it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(acc_empty(buf));
        }
        if (live) {
          __half *dst = part == 0 ? p.left + static_cast<int64_t>(i) * p.pitch + sq
                                  : p.right + static_cast<int64_t>(i) * C * p.pitch + sq;
          const int64_t stride = part == 0 ? p.rows * p.pitch : p.pitch;
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            const int col = part * 32 + k;
            const float y = fmaf(__uint_as_float(v[k]), vsm[col], vsm[64 + col]) * mk;
            dst[k * stride] = __float2half_rn(y);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 128);
  }
}

// ---- outer products: outer[(i, j)][a*32 + b] = 2^-shift sum_s left[s][i][a] right[s][j][b] ----
constexpr int OBM = 128, OBN = 256, OBK = 64, OSTAGES = 4, OTHREADS = 192;
constexpr uint32_t OA_BYTES = OBM * 128, OB_BYTES = OBN * 128, OSTAGE = OA_BYTES + OB_BYTES;
constexpr uint32_t OOFF_BAR = OSTAGES * OSTAGE;
constexpr uint32_t OSMEM = OOFF_BAR + 256 + 1024;

struct OuterArgs {
  __half *outer;  // [(i - i_begin) * n + j][1024], or [..][3 * 1024] when split
  int n, i_begin, i_count, tiles_j, k_blocks, total_tiles;
  int rows_b;     // residues per block of the right operand ([blocks][S][rows_b][c]): n unless sharded
  float scale;
  int split;  // f32 precision mode: rows [f16(v) | f16(v) | f16(v - f16(v))] for the K-tripled output GEMM
  unsigned int *err;
};

__global__ void __launch_bounds__(OTHREADS, 1)
    outer_kernel(const __grid_constant__ CUtensorMap lmap, const __grid_constant__ CUtensorMap rmap,
                 const OuterArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + OOFF_BAR;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (OSTAGES + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * OSTAGES + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * OSTAGES + 2 + b); };
  const uint32_t drain = bar0 + 8u * (2 * OSTAGES + 4);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OOFF_BAR + 128);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OOFF_BAR + 136);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < OSTAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), 4);
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
    if (lane == 0) {
      tma_prefetch_map(&lmap);
      tma_prefetch_map(&rmap);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
        const int ti = t / p.tiles_j, tj = t - ti * p.tiles_j;
        const int i0 = p.i_begin + ti * 4, j0 = tj * 8;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % OSTAGES;
          if (!mbar_wait(empty(s), ((it / OSTAGES) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t dst = sbase + s * OSTAGE;
          mbar_arrive_expect_tx(full(s), OSTAGE);
          // [64 s rows][64 (i, a) elements] boxes: 2 for the 128-wide A tile, 4 for the 256-wide B tile
          for (int b = 0; b < 2; ++b) tma_load_3d(dst + b * 8192, &lmap, full(s), i0 * C + b * 64, kb * OBK, 0);
          const int jb = j0 / p.rows_b, jl = j0 - jb * p.rows_b;  // 8 residues never straddle two blocks
          for (int b = 0; b < 4; ++b)
            tma_load_3d(dst + OA_BYTES + b * 8192, &rmap, full(s), jl * C + b * 64, kb * OBK, jb);
        }
      }
      for (int j = std::max(0, it - OSTAGES); j < it; ++j) mbar_wait_drain(full(j % OSTAGES), (j / OSTAGES) & 1, p.err);
    }
  } else if (warp == 1) {
      // both operands MN-major: 64-element MN blocks 8 KB apart, 8-row K groups 1 KB apart
    constexpr uint32_t kIdesc = idesc_f16_f32(OBM, OBN) | (1u << 15) | (1u << 16);
    const uint64_t a_desc = sdesc_mn_sw128(sbase, 8192, 1024);
    int it = 0, tile_it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x, ++tile_it) {
      const int buf = tile_it & 1;
      if (!warp_wait(acc_empty(buf), ((tile_it >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitMma)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * OBN;
      for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
        const int s = it % OSTAGES;
        if (!warp_wait(full(s), (it / OSTAGES) & 1, abort_flag, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = desc_add(a_desc, s * OSTAGE), bd = desc_add(ad, OA_BYTES);
        if (kb == 0)
          umma_first(d, ad, bd, kIdesc);
        else
          umma_acc(d, ad, bd, kIdesc);
#pragma unroll
        for (int ks = 1; ks < OBK / 16; ++ks) umma_acc(d, desc_add(ad, ks * 2048), desc_add(bd, ks * 2048), kIdesc);
        umma_commit(empty(s));
      }
      if (ok) umma_commit(acc_full(buf));
    }
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else {
    // TMEM lane = (i_local, a) with i_local = this warp's quarter, a = lane;
    // columns = (j_local, b).  Each (pair, a) is 32 contiguous f16 of the row.
    const int q = warp & 3;
    int tile_it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++tile_it) {
      const int ti = t / p.tiles_j, tj = t - ti * p.tiles_j;
      const int i = p.i_begin + ti * 4 + q, j0 = tj * 8;
      const int buf = tile_it & 1;
      if (!warp_wait(acc_full(buf), (tile_it >> 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * OBN;
      const bool i_ok = i < p.i_begin + p.i_count;
#pragma unroll 1
      for (int jl = 0; jl < 8; ++jl) {
        uint32_t v[32];
        tmem_ld32(taddr + jl * 32, v);
        tmem_ld_wait();
        const int j = j0 + jl;
        if (!i_ok || j >= p.n) continue;
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 32; c += 2)
          pk[c >> 1] = pack_half2(__uint_as_float(v[c]) * p.scale, __uint_as_float(v[c + 1]) * p.scale);
        const int64_t pitch = p.split ? 3 * C * C : C * C;
        uint4 *dst = reinterpret_cast<uint4 *>(p.outer + (static_cast<int64_t>(i - p.i_begin) * p.n + j) * pitch +
                                              lane * C);
#pragma unroll
        for (int w = 0; w < 4; ++w) dst[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
        if (p.split) {
          uint32_t lo[16];
#pragma unroll
          for (int c = 0; c < 32; c += 2) {
            const __half2 h = *reinterpret_cast<const __half2 *>(&pk[c >> 1]);
            lo[c >> 1] = pack_half2(__uint_as_float(v[c]) * p.scale - __low2float(h),
                                    __uint_as_float(v[c + 1]) * p.scale - __high2float(h));
          }
          uint4 *d1 = dst + (C * C) / 8, *d2 = dst + (2 * C * C) / 8;
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            d1[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
            d2[w] = make_uint4(lo[4 * w], lo[4 * w + 1], lo[4 * w + 2], lo[4 * w + 3]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(buf));
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- the outer products and the output projection in one kernel ----
// A tile is 128 residues i (the TMEM lanes) x J residues j (J = 3 when the
// tile's right operand fits beside the left ring, S <= 512; else 2).  For each
// outer channel a (a "slice") the tensor core forms
//   D1[i][(j, b)] = sum_s left[a][i][s] right[j][b][s]      (M 128, N 32 J, K S)
// with left streamed through a ring and the tile's right operand resident in
// shared memory, both K-major (sequences contiguous: MN-major operands run the
// tensor core several times slower at this N).  Worker warps round D1 * 2^-k
// to f16 (one warp per lane quarter and residue j, 32 columns each) into A2,
// and the tensor core multiplies it, read as an A operand from TMEM (or, for
// the third residue of a three-residue tile, from shared memory), by the 32
// rows of W_o that belong to channel a:
//   D2_j[i][z] += A2_j[i][b] W_o[a*32 + b][z]                (M 128, N c_z, K 32)
// The outer products never leave the SM.  After the 32 slices the same
// workers apply the column scales (which carry 2^k back), b_o, 1/(eps + count)
// and the residual, and write the pair rows, while the next tile's first outer
// products run.  D2 sums K = (a, b) in ascending 16-wide steps, as the
// two-kernel path does, from the same f16 operand values.
//
// TMEM (512 columns): D2_j at 128 j.  The output MMAs of slice g are issued
// behind the outer products of slice g + 1.  J = 2: D1 double-buffered at 256
// and 320, A2 at 384 and 416.  J = 3: D1 (96 columns) single at 384, released
// to the outer products of slice g + 1 as soon as the workers have loaded it;
// A2_0 and A2_1 at 480 and 496 and A2_2, for which TMEM has no room left, in
// an 8 KB shared-memory tile (64B-swizzled, K-major) read by an SS MMA.
// Each streamed byte of left serves 32 J outputs per sequence, so J = 3 cuts
// the left traffic per pair (the kernel's bound, through L2) by a third.
// Tiles are dealt to CTAs in contiguous runs (j-group major), so a CTA reloads
// the resident right operand only when its j group changes.
constexpr int FTHREADS = 448;  // warp 0 TMA, 1 MMA, 2-13 workers (slice conversion, output epilogue)
constexpr int FLST_MAX = 8;    // left ring: [128 i][64 s] f16 per stage, as many as shared memory holds
constexpr uint32_t FL_STAGE = 16384, FW_STAGE = 8192;  // W_o: one channel's 32 rows x c_z, 64B-swizzled
constexpr uint32_t kD2Col = 0;
constexpr uint32_t kFusedSmemLimit = 232448;  // 227 KB of dynamic shared memory per CTA
constexpr uint32_t kFusedBarBytes = 512;

template <int J>
struct FusedCfg {
  static constexpr uint32_t kRBlock = J * 32 * 128;            // resident right: bytes per 64-sequence block
  static constexpr int kNB = J == 2 ? 2 : 1;                    // D1 buffers
  static constexpr uint32_t kD1Col = J == 2 ? 256 : 384;
  static constexpr uint32_t kA2Col = J == 2 ? 384 : 480;
  static constexpr uint32_t kD1Stride = 64, kA2Stride = 32;     // between buffers (J = 2)
  static constexpr uint32_t kA2J = 16;                          // between the A2 blocks of residues j
  static constexpr int kA2Tmem = 2;  // residues whose A2 is in TMEM (J = 3: the third's is in shared memory)
};

// Shared-memory map: right (resident) | left ring | W_o ring (2) | A2 tile of the
// third residue (J = 3: [128 i][32 b] f16, 64B-swizzled) | barriers.
__host__ __device__ constexpr uint32_t fused_off_l(int k_blocks, int j) {
  return static_cast<uint32_t>(k_blocks) * j * 32u * 128u;
}
__host__ __device__ constexpr uint32_t fused_off_w(int k_blocks, int j, int lst) {
  return fused_off_l(k_blocks, j) + static_cast<uint32_t>(lst) * FL_STAGE;
}
constexpr uint32_t kFusedA2Bytes = 128 * 64;
__host__ __device__ constexpr uint32_t fused_off_a2(int k_blocks, int j, int lst) {
  return fused_off_w(k_blocks, j, lst) + 2 * FW_STAGE;
}
__host__ __device__ constexpr uint32_t fused_off_bar(int k_blocks, int j, int lst) {
  return fused_off_a2(k_blocks, j, lst) + (j == 3 ? kFusedA2Bytes : 0u);
}
__host__ __device__ constexpr uint32_t fused_smem(int k_blocks, int j, int lst) {
  return fused_off_bar(k_blocks, j, lst) + kFusedBarBytes + 1024;
}
// Left stages that fit beside the resident right operand (0 when fewer than 2 do).
__host__ __device__ constexpr int fused_stages(int k_blocks, int j) {
  int lst = FLST_MAX;
  while (lst > 0 && fused_smem(k_blocks, j, lst) > kFusedSmemLimit) --lst;
  return lst >= 2 ? lst : 0;
}
constexpr int kFusedMaxKBlocks = 16;  // S <= 1024 (J = 2); J = 3 needs S <= 512

// Tile t = jg * n_ib + r is residue block (r + jg) mod n_ib of j group jg: CTAs
// working on different j groups at the same moment stream different blocks of left.
__device__ __forceinline__ int fused_tile_ib(int t, int jg, int n_ib) {
  int ib = t - jg * n_ib + jg % n_ib;
  return ib >= n_ib ? ib - n_ib : ib;
}

struct FusedArgs {
  void *out;                   // this rank's pair rows [rows][n][cz]
  const float *wscale, *bias;  // per output column (n_out entries)
  const float *rowscale;       // [rows][n]: 1 / (eps + count)
  int64_t n, rows;
  int cz, n_out, n_ib, total_tiles, per_cta, k_blocks;
  int lst;                     // left ring stages
  float scale;                 // 2^-k applied to D1 before rounding
  int residual, vector_out;
  int out_bytes;               // bytes per output element
  unsigned int *err;
};

template <typename OT, int J>
__global__ void __launch_bounds__(FTHREADS, 1)
    fused_kernel(const __grid_constant__ CUtensorMap lmap, const __grid_constant__ CUtensorMap rmap,
                 const __grid_constant__ CUtensorMap wmap, const FusedArgs p) {
  using Cfg = FusedCfg<J>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const int lst = p.lst;
  const uint32_t s_r = sbase, s_l = sbase + fused_off_l(p.k_blocks, J), s_w = sbase + fused_off_w(p.k_blocks, J, lst);
  const uint32_t bar0 = sbase + fused_off_bar(p.k_blocks, J, lst);
  auto l_full = [&](int s) { return bar0 + 8u * s; };
  auto l_empty = [&](int s) { return bar0 + 8u * (FLST_MAX + s); };
  auto w_full = [&](int s) { return bar0 + 8u * (2 * FLST_MAX + s); };
  auto w_empty = [&](int s) { return bar0 + 8u * (2 * FLST_MAX + 2 + s); };
  auto d1_full = [&](int b) { return bar0 + 8u * (2 * FLST_MAX + 4 + b); };
  auto a2_full = [&](int b) { return bar0 + 8u * (2 * FLST_MAX + 6 + b); };
  auto a2_empty = [&](int b) { return bar0 + 8u * (2 * FLST_MAX + 8 + b); };
  const uint32_t r_full = bar0 + 8u * (2 * FLST_MAX + 10), r_empty = r_full + 8u, d2_full = r_full + 16u,
                 d2_empty = r_full + 24u, drain = r_full + 32u;
  const uint32_t d1_free = r_full + 40u;  // J = 3: the workers have loaded D1 (32 barriers: 256 bytes)
  const uint32_t s_a2 = sbase + fused_off_a2(p.k_blocks, J, lst);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + fused_off_bar(p.k_blocks, J, lst) + 256);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + fused_off_bar(p.k_blocks, J, lst) + 264);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;
  const int t_begin = blockIdx.x * p.per_cta;
  const int t_end = min(p.total_tiles, t_begin + p.per_cta);

  if (threadIdx.x == 0) {
    for (int s = 0; s < lst; ++s) {
      mbar_init(l_full(s), 1);
      mbar_init(l_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(w_full(b), 1);
      mbar_init(w_empty(b), 1);
      mbar_init(d1_full(b), 1);
      mbar_init(a2_full(b), 4 * J);
      mbar_init(a2_empty(b), 1);
    }
    mbar_init(r_full, 1);
    mbar_init(r_empty, 1);
    mbar_init(d2_full, 1);
    mbar_init(d2_empty, 4 * J);
    mbar_init(d1_free, 4 * J);
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
    if (lane == 0) {
      tma_prefetch_map(&lmap);
      tma_prefetch_map(&rmap);
      tma_prefetch_map(&wmap);
      int ls = 0, lph = 0, lcount = 0, wq = 0, rq = 0, prev_jg = -1;
      bool ok = true;
      const uint32_t w_bytes = static_cast<uint32_t>(p.n_out) * 64u;
      for (int t = t_begin; ok && t < t_end; ++t) {
        const int jg = t / p.n_ib, ib = fused_tile_ib(t, jg, p.n_ib);
        if (jg != prev_jg) {
          // the resident right operand of j = J jg .. J jg + J - 1: rows 32 J jg .. of [n * c][S]
          if (rq > 0 && !mbar_wait(r_empty, (rq - 1) & 1, abort_flag, p.err, kErrWaitProducer)) break;
          mbar_arrive_expect_tx(r_full, static_cast<uint32_t>(p.k_blocks) * Cfg::kRBlock);
          for (int kb = 0; kb < p.k_blocks; ++kb)
            tma_load_3d(s_r + kb * Cfg::kRBlock, &rmap, r_full, kb * 64, 32 * J * jg, 0);
          ++rq;
          prev_jg = jg;
        }
        for (int a = 0; ok && a < C; ++a) {
          for (int kb = 0; kb < p.k_blocks; ++kb) {
            if (!mbar_wait(l_empty(ls), lph ^ 1, abort_flag, p.err, kErrWaitProducer)) {
              ok = false;
              break;
            }
            const uint32_t dst = s_l + ls * FL_STAGE;
            mbar_arrive_expect_tx(l_full(ls), FL_STAGE);
            tma_load_3d(dst, &lmap, l_full(ls), kb * 64, 128 * ib, a);  // [128 residues][64 sequences]
            ++lcount;
            if (++ls == lst) {
              ls = 0;
              lph ^= 1;
            }
          }
          if (!ok) break;
          {  // W_o rows of channel a: one [n_out][32] K-major tile, used by the output MMAs that
             // follow the next slice's outer products, so it is loaded after this slice's left
            const int ws = wq & 1;
            if (!mbar_wait(w_empty(ws), ((wq >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(w_full(ws), w_bytes);
            tma_load_3d(s_w + ws * FW_STAGE, &wmap, w_full(ws), (a & 1) * 32, 0, a >> 1);
            ++wq;
          }
        }
      }
      // loads still in flight (all consumed unless a role gave up)
      for (int j = max(0, lcount - lst); j < lcount; ++j) mbar_wait_drain(l_full(j % lst), (j / lst) & 1, p.err);
      for (int j = max(0, wq - 2); j < wq; ++j) mbar_wait_drain(w_full(j & 1), (j >> 1) & 1, p.err);
      if (rq > 0) mbar_wait_drain(r_full, (rq - 1) & 1, p.err);
    }
  } else if (warp == 1) {
    // MMA issue: the whole warp runs the loop (warp-uniform waits and running
    // descriptors) and one elected lane issues each instruction.  Every operand
    // is K-major: a 16-sequence step is 32 bytes (2 descriptor units) along the
    // 128-byte rows; a left stage is 16 KB (1024 units).
    const uint32_t idesc1 = idesc_f16_f32(128, 32 * J);
    const uint32_t idesc2 = idesc_f16_f32(128, p.n_out);  // A in TMEM
    const uint64_t l_base = sdesc_k_sw128(s_l), r_base = sdesc_k_sw128(s_r), w_base = sdesc_k_sw64(s_w);
    uint64_t l_desc = l_base;
    int ls = 0, lph = 0, wq = 0, rq = 0, prev_jg = -1, tile_it = 0;
    uint32_t g = 0;  // slices issued, over all tiles
    bool ok = true;
    // D2_j += A2_j(slice gp) W_o(channel a)
    auto outputs = [&](uint32_t gp, int a) -> bool {
      const int bp = gp % Cfg::kNB, ws = wq & 1;
      if (a == 0 && !warp_wait(d2_empty, (tile_it & 1) ^ 1, abort_flag, p.err, kErrWaitMma)) return false;
      if (!warp_wait(a2_full(bp), (gp / Cfg::kNB) & 1, abort_flag, p.err, kErrWaitMma)) return false;
      if (!warp_wait(w_full(ws), (wq >> 1) & 1, abort_flag, p.err, kErrWaitMma)) return false;
      tc_fence_after();
      const uint64_t bd = w_base + ws * (FW_STAGE >> 4);
      const uint32_t a2 = tmem + Cfg::kA2Col + bp * Cfg::kA2Stride;
#pragma unroll
      for (int j = 0; j < J; ++j) {
        if (j < Cfg::kA2Tmem) {
          if (a == 0)
            umma_ts_first(tmem + kD2Col + 128 * j, a2 + Cfg::kA2J * j, bd, idesc2);
          else
            umma_ts_acc(tmem + kD2Col + 128 * j, a2 + Cfg::kA2J * j, bd, idesc2);
          umma_ts_acc(tmem + kD2Col + 128 * j, a2 + Cfg::kA2J * j + 8, bd + 2, idesc2);
        } else {  // J = 3, third residue: A2 from the shared-memory tile
          const uint64_t ad = sdesc_k_sw64(s_a2);
          if (a == 0)
            umma_first(tmem + kD2Col + 128 * j, ad, bd, idesc2);
          else
            umma_acc(tmem + kD2Col + 128 * j, ad, bd, idesc2);
          umma_acc(tmem + kD2Col + 128 * j, ad + 2, bd + 2, idesc2);
        }
      }
      umma_commit(a2_empty(bp));
      umma_commit(w_empty(ws));
      ++wq;
      return true;
    };
    for (int t = t_begin; ok && t < t_end; ++t, ++tile_it) {
      const int jg = t / p.n_ib;
      if (jg != prev_jg) {
        if (!warp_wait(r_full, rq & 1, abort_flag, p.err, kErrWaitMma)) break;
        ++rq;
        prev_jg = jg;
      }
      for (int a = 0; a < C; ++a, ++g) {
        if (J == 3 && g > 0 && !warp_wait(d1_free, ((g - 1) & 1), abort_flag, p.err, kErrWaitMma)) {
          ok = false;  // the single D1 is free once the workers have loaded slice g - 1's
          break;
        }
        const uint32_t d1 = tmem + Cfg::kD1Col + (g % Cfg::kNB) * Cfg::kD1Stride;
        uint64_t r_desc = r_base;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!warp_wait(l_full(ls), lph, abort_flag, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (kb == 0)
            umma_first(d1, l_desc, r_desc, idesc1);
          else
            umma_acc(d1, l_desc, r_desc, idesc1);
          umma_acc(d1, l_desc + 2, r_desc + 2, idesc1);
          umma_acc(d1, l_desc + 4, r_desc + 4, idesc1);
          umma_acc(d1, l_desc + 6, r_desc + 6, idesc1);
          umma_commit(l_empty(ls));
          r_desc += Cfg::kRBlock >> 4;
          l_desc += FL_STAGE >> 4;
          if (++ls == lst) {
            ls = 0;
            lph ^= 1;
            l_desc = l_base;
          }
        }
        if (!ok) break;
        umma_commit(d1_full(g % Cfg::kNB));
        if (a > 0 && !outputs(g - 1, a - 1)) {
          ok = false;
          break;
        }
      }
      if (!ok || !outputs(g - 1, C - 1)) break;
      umma_commit(d2_full);
      if (t + 1 < t_end && (t + 1) / p.n_ib != jg) umma_commit(r_empty);
    }
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else {
    // ---- workers: warp (q, jw) owns TMEM lanes 32 q .. 32 q + 31 of residue jw's columns ----
    // Per slice it converts D1_jw (f32) to A2_jw (f16 pairs, times 2^-k); at the end of a
    // tile it drains D2_jw: column scales (which carry 2^k back), b_o, 1 / (eps + count) and
    // the residual, written to the pair rows.  Twelve warps share each slice's conversion,
    // so the tensor pipe waits for 32 columns per lane, not 32 J.
    const int q = warp & 3, jw = (warp - 2) >> 2;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const int chunks = p.n_out / 32;
    if (jw < J) {
      uint32_t g = 0;
      int tile_it = 0;
      bool ok = true;
      for (int t = t_begin; ok && t < t_end; ++t, ++tile_it) {
        for (int a = 0; a < C; ++a, ++g) {
          const int b = g % Cfg::kNB;
          if (!warp_wait(d1_full(b), (g / Cfg::kNB) & 1, abort_flag, p.err, kErrWaitEpilogue) ||
              (J == 2 && !warp_wait(a2_empty(b), ((g >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitEpilogue))) {
            ok = false;
            break;
          }
          tc_fence_after();
          uint32_t v[32], pk[16];
          tmem_ld32(tmem + lane_off + Cfg::kD1Col + b * Cfg::kD1Stride + 32 * jw, v);
          tmem_ld_wait();
          if (J == 3) {  // D1 is loaded: the next slice's outer products may overwrite it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d1_free);
          }
#pragma unroll
          for (int c = 0; c < 16; ++c)
            pk[c] = pack_half2(__uint_as_float(v[2 * c]) * p.scale, __uint_as_float(v[2 * c + 1]) * p.scale);
          // J = 3: the previous slice's output MMAs have read A2
          if (J == 3 && g > 0) {
            if (!warp_wait(a2_empty(0), (g - 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) {
              ok = false;
              break;
            }
            tc_fence_after();
          }
          if (jw < Cfg::kA2Tmem) {
            tmem_st16(tmem + lane_off + Cfg::kA2Col + b * Cfg::kA2Stride + Cfg::kA2J * jw, pk);
            tmem_st_wait();
          } else {
            // row i = 32 q + lane of the [128][32] f16 tile, 64 bytes in four 16-byte chunks,
            // chunk c stored at c ^ ((i >> 1) & 3) (the 64-byte swizzle)
            const int i = q * 32 + lane;
            uint8_t *row = smem + fused_off_a2(p.k_blocks, J, lst) + i * 64;
#pragma unroll
            for (int c = 0; c < 4; ++c)
              *reinterpret_cast<uint4 *>(row + ((c ^ ((i >> 1) & 3)) << 4)) =
                  make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            fence_async_smem();
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(a2_full(b));
          if (a == C - 4 && p.residual) {
            // the pair row this thread adds into at the end of the tile: into L2 ahead of time
            const int jg = t / p.n_ib, ib = fused_tile_ib(t, jg, p.n_ib);
            const int64_t i = static_cast<int64_t>(ib) * 128 + q * 32 + lane, j = static_cast<int64_t>(J) * jg + jw;
            if (i < p.rows && j < p.n) {
              const char *row = reinterpret_cast<const char *>(p.out) + (i * p.n + j) * p.cz * p.out_bytes;
              for (int off = 0; off < p.cz * p.out_bytes; off += 128)
                asm volatile("prefetch.global.L2 [%0];" ::"l"(row + off));
            }
          }
        }
        if (!ok) break;
        // ---- output epilogue of this tile: D2_jw, lanes 32 q .. ----
        const int jg = t / p.n_ib, ib = fused_tile_ib(t, jg, p.n_ib);
        const int64_t i = static_cast<int64_t>(ib) * 128 + q * 32 + lane;
        if (!warp_wait(d2_full, tile_it & 1, abort_flag, p.err, kErrWaitEpilogue)) break;
        tc_fence_after();
        const int64_t j = static_cast<int64_t>(J) * jg + jw;
        const bool row_ok = i < p.rows && j < p.n;
        const float rs = row_ok ? p.rowscale[i * p.n + j] : 0.f;
        OT *orow = static_cast<OT *>(p.out) + (i * p.n + j) * p.cz;
        for (int ch = 0; ch < chunks; ++ch) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + kD2Col + jw * 128 + ch * 32, v);
          tmem_ld_wait();
          if (ch == chunks - 1) {  // D2 is free for the next tile once every lane has read it
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(d2_empty);
          }
          const int c0 = ch * 32;
          if (!row_ok || c0 >= p.cz) continue;
          float y[32];
          const float4 *sc = reinterpret_cast<const float4 *>(p.wscale + c0);
          const float4 *bi = reinterpret_cast<const float4 *>(p.bias + c0);
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const float4 s4 = __ldg(sc + i4), b4 = __ldg(bi + i4);
            y[4 * i4 + 0] = fmaf(__uint_as_float(v[4 * i4 + 0]), s4.x, b4.x) * rs;
            y[4 * i4 + 1] = fmaf(__uint_as_float(v[4 * i4 + 1]), s4.y, b4.y) * rs;
            y[4 * i4 + 2] = fmaf(__uint_as_float(v[4 * i4 + 2]), s4.z, b4.z) * rs;
            y[4 * i4 + 3] = fmaf(__uint_as_float(v[4 * i4 + 3]), s4.w, b4.w) * rs;
          }
          store_out32<OT>(orow, c0, p.cz, y, p.vector_out, p.residual);
        }
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

}  // namespace opm

using namespace opm;

OpmLayout opm_layout(int64_t s, int64_t n, int64_t cm, int64_t c, int64_t cz, int64_t row_block, int64_t rows,
                     int64_t row0, bool split) {
  OpmLayout L;
  // f32 precision mode: every operand an f16 hi / lo pair, each GEMM's K tripled (hi hi + hi lo + lo hi)
  L.split = split;
  const int64_t kx = split ? 3 : 1;
  L.s = s;
  L.n = n;
  L.rows = (rows <= 0 || rows > n) ? n : rows;
  L.row0 = row0;
  L.cm = cm;
  L.c = c;
  L.cz = cz;
  L.cmp = align_up(cm, 64);
  // Residue block: the outer scratch stays within 256 MiB unless asked otherwise; a multiple of 4.
  int64_t rb = row_block > 0 ? row_block : std::max<int64_t>(4, (int64_t(256) << 20) / (n * c * c * 2 * kx));
  rb = std::min<int64_t>(align_up(std::max<int64_t>(rb, 1), 4), align_up(L.rows, 4));
  L.block_rows = rb;
  int k = 0;
  while ((int64_t(1) << k) < s) ++k;
  L.out_shift = k;
  // One kernel for the outer products and the output projection when the
  // right operand of a tile fits in shared memory and c_z in one MMA.
  L.fused = !split && c == C && align_up(s, 64) / 64 <= kFusedMaxKBlocks && cz <= 128;
  L.seq_pitch = L.fused ? align_up(s, 8) : 0;
  const int64_t lr_cols = linear_cols_pad(2 * c), o_cols = linear_cols_pad(cz), o_inner = align_up(c * c, 64);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.off_wlr = take((size_t)kx * L.cmp * lr_cols * 2);
  L.off_wlr_scale = take((size_t)lr_cols * 4);
  L.off_wlr_bias = take((size_t)lr_cols * 4);
  L.off_wo = take((size_t)kx * o_inner * o_cols * 2);
  L.off_wo_scale = take((size_t)o_cols * 4);
  L.off_wo_bias = take((size_t)o_cols * 4);
  L.off_ln = take((size_t)L.cmp * 2 * 4);
  L.off_xn = take((size_t)kx * s * L.rows * L.cmp * 2);
  L.off_mask = take((size_t)s * L.rows * 4);
  const int64_t seq_span = L.fused ? L.seq_pitch : s;
  L.off_left = take((size_t)kx * seq_span * c * L.rows * 2);
  L.off_right = take((size_t)kx * seq_span * n * c * 2);  // every rank's block: [ranks][S][rows][c], or [n][c][pitch]
  L.off_rowscale = take((size_t)L.rows * n * 4);
  L.off_outer = take(L.fused ? 0 : (size_t)kx * rb * n * c * c * 2);
  L.off_stage = L.off_xn;
  L.total = std::max(off, align_up(L.off_stage + (size_t)(2 * cm + 2 * (cm * c + c) + cz) * 4, 256));
  return L;
}

namespace {

template <typename OT, int J>
af2_status launch_fused_t(af2_ctx *ctx, const CUtensorMap &lmap, const CUtensorMap &rmap, const CUtensorMap &wmap,
                          const FusedArgs &a, int grid, cudaStream_t stream) {
  const uint32_t smem = fused_smem(a.k_blocks, J, a.lst);
  cudaError_t e = cudaFuncSetAttribute(fused_kernel<OT, J>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "fused OPM kernel attributes");
  LaunchScope scope(ctx, stream, kProfOpmFused);
  fused_kernel<OT, J><<<grid, FTHREADS, smem, stream>>>(lmap, rmap, wmap, a);
  e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "fused OPM kernel launch");
}

// The outer products and output projection of this rank's rows, one launch.
af2_status fused_launch(af2_ctx *ctx, const OpmLayout &L, uint8_t *ws, const uint8_t *wp, const __half *right_full,
                        int residual, void *out, int out_dtype, cudaStream_t stream) {
  const int64_t s = L.s, n = L.n, c = L.c, cz = L.cz, rows = L.rows;
  const int64_t o_cols = linear_cols_pad(cz), o_inner = align_up(c * c, 64);
  const int k_blocks = (int)((s + 63) / 64);
  // three residues j per tile when their right operand fits beside the left ring, else two;
  // AF2_OPM_TILE_RESIDUES=2 selects two where three fit (S = 512, N = 1024: 2.15 ms
  // against 1.49 ms with three, one B200)
  const int J = fused_stages(k_blocks, 3) >= 4 && tuning_override("AF2_OPM_TILE_RESIDUES", 3) != 2 ? 3 : 2;
  CUtensorMap lmap, rmap, wmap;
  // K-major, sequences contiguous (zero past S):
  // left [c][rows][pitch]: boxes of 64 sequences x 128 residues of one channel
  // right [n][c][pitch]: boxes of 64 sequences x 32 J rows (J residues x 32 channels)
  // W_o [c*c / 64][o_cols][64]: the 32 rows of one channel a per box (64B-swizzled)
  const uint64_t pitch = L.seq_pitch;
  if (!encode_map_3d(&lmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_left, s, rows, c, pitch * 2,
                     (uint64_t)rows * pitch * 2, 64, 128, 1, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&rmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, right_full, s, n * c, 1, pitch * 2,
                     (uint64_t)n * c * pitch * 2, 64, (uint32_t)(32 * J), 1, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&wmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, wp + L.off_wo, 64, o_cols, o_inner / 64, 128,
                     (uint64_t)o_cols * 128, 32, (uint32_t)o_cols, 1, CU_TENSOR_MAP_SWIZZLE_64B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the fused OPM operands");
  FusedArgs a{};
  a.out = out;
  a.wscale = reinterpret_cast<const float *>(wp + L.off_wo_scale);
  a.bias = reinterpret_cast<const float *>(wp + L.off_wo_bias);
  a.rowscale = reinterpret_cast<const float *>(ws + L.off_rowscale);
  a.n = n;
  a.rows = rows;
  a.cz = (int)cz;
  a.n_out = (int)o_cols;
  a.n_ib = (int)((rows + 127) / 128);
  a.total_tiles = a.n_ib * (int)((n + J - 1) / J);
  a.per_cta = (a.total_tiles + ctx->sm_count - 1) / ctx->sm_count;
  a.k_blocks = k_blocks;
  a.lst = fused_stages(k_blocks, J);
  a.scale = std::ldexp(1.f, -L.out_shift);
  a.residual = residual;
  {
    const size_t ob = out_dtype == AF2_F32 ? 4 : 2;
    a.vector_out = reinterpret_cast<uintptr_t>(out) % 16 == 0 && (cz * ob) % 16 == 0;
    a.out_bytes = (int)ob;
  }
  a.err = ctx->err_word;
  const int grid = (a.total_tiles + a.per_cta - 1) / a.per_cta;
  auto run = [&](auto jtag) {
    constexpr int JJ = decltype(jtag)::value;
    if (out_dtype == AF2_F16) return launch_fused_t<__half, JJ>(ctx, lmap, rmap, wmap, a, grid, stream);
    if (out_dtype == AF2_BF16) return launch_fused_t<__nv_bfloat16, JJ>(ctx, lmap, rmap, wmap, a, grid, stream);
    return launch_fused_t<float, JJ>(ctx, lmap, rmap, wmap, a, grid, stream);
  };
  return J == 3 ? run(std::integral_constant<int, 3>{}) : run(std::integral_constant<int, 2>{});
}

}  // namespace

af2_status opm_launch(af2_ctx *ctx, const OpmLayout &L, const void *m, int m_dtype, const float *mask,
                      const float *packed, double ln_eps, double norm_eps, int residual, void *out, int out_dtype,
                      void *workspace, cudaStream_t stream, const OpmExchange *exchange, const af2_matrix *tensors) {
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int64_t s = L.s, n = L.n, cm = L.cm, c = L.c, cz = L.cz, rows = L.rows;
  const int rank = exchange ? exchange->rank : 0;
  // packOuterProductMeanWeights order (outer-product-mean.ts:68-72).
  const float *ln_w = nullptr, *ln_b = nullptr, *lw = nullptr, *lb = nullptr, *rw = nullptr, *rb = nullptr;
  const float *ow = nullptr, *ob = nullptr;
  if (!tensors) {
    ln_w = packed, ln_b = ln_w + cm, lw = ln_b + cm, lb = lw + cm * c, rw = lb + c, rb = rw + cm * c;
    ow = rb + c, ob = ow + c * c * cz;
  }
  const int64_t lr_cols = linear_cols_pad(2 * c), o_cols = linear_cols_pad(cz), o_inner = align_up(c * c, 64);
  af2_status st;
  // 16-bit MSA, fused layouts: LayerNorm and projection in one kernel (gamma and beta folded
  // into the projection's weights and biases)
  const bool lnproj = L.fused && m_dtype != AF2_F32 && cm % 8 == 0 && L.cmp <= 256 &&
                      reinterpret_cast<uintptr_t>(m) % 16 == 0;
  // the MSA's residue columns: all n, or only this rank's rows when the exchange says so
  const bool m_local = exchange && exchange->m_local;
  const int64_t m_cols = m_local ? rows : n, m_col0 = m_local ? 0 : L.row0;
  const int64_t kx = L.split ? 3 : 1;
  // the prepared weights: the layout's prefix [0, off_xn), in the weight cache or the workspace
  WeightKey key;
  key.kind = tensors ? kWeightsOpmTensors : kWeightsOpm;
  key.ptr[0] = packed;
  if (tensors)
    for (int t = 0; t < 8; ++t) key.ptr[t] = tensors[t].values, key.ptr[8 + t] = tensors[t].scales;
  const int64_t dims[7] = {cm, c, cz, L.out_shift, lnproj ? 1 : 0, L.split ? 1 : 0, L.cmp};
  for (int i = 0; i < 7; ++i) key.dim[i] = dims[i];
  PreparedRegion pw;
  if ((st = prepared_region(ctx, key, L.off_xn, ws, true, &pw)) != AF2_OK) return st;
  uint8_t *wp = pw.base;
  float *wlr_scale = reinterpret_cast<float *>(wp + L.off_wlr_scale), *wlr_bias = reinterpret_cast<float *>(wp + L.off_wlr_bias);
  float *wo_scale = reinterpret_cast<float *>(wp + L.off_wo_scale), *wo_bias = reinterpret_cast<float *>(wp + L.off_wo_bias);
  float *ln = reinterpret_cast<float *>(wp + L.off_ln);
  // ---- weights ----
  if (tensors && pw.fresh) {
    // the small tensors in f32: f32 ones as given, q8 ones decoded into the staging region
    // (the products code x f16 scale are exact in f32, so the decode is the reference's own)
    float *stage = reinterpret_cast<float *>(ws + L.off_stage);
    const float **dst[7] = {&ln_w, &ln_b, &lw, &lb, &rw, &rb, &ob};
    const int src[7] = {0, 1, 2, 3, 4, 5, 7};
    const int64_t count[7] = {cm, cm, cm * c, c, cm * c, c, cz};
    for (int i = 0; i < 7; ++i) {
      const af2_matrix &t = tensors[src[i]];
      if (t.format == AF2_WEIGHTS_F32) {
        *dst[i] = static_cast<const float *>(t.values);
      } else {
        if ((st = dequant_launch(ctx, t, 1, count[i], stage, stream)) != AF2_OK) return st;
        *dst[i] = stage;
      }
      stage += count[i];
    }
  }
  const af2_matrix left_m{AF2_WEIGHTS_F32, 0, lw, nullptr}, right_m{AF2_WEIGHTS_F32, 0, rw, nullptr};
  const af2_matrix out_m = tensors ? tensors[6] : af2_matrix{AF2_WEIGHTS_F32, 0, ow, nullptr};
  VectorSegments vs{};
  vs.add(lb, c, c, wlr_bias);
  vs.add(rb, c, lr_cols - c, wlr_bias + c);
  vs.add(ob, cz, o_cols, wo_bias);
  vs.add(ln_w, cm, L.cmp, ln);
  vs.add(ln_b, cm, L.cmp, ln + L.cmp);
  if (lr_cols > 2 * c) vs.add(nullptr, 0, lr_cols - 2 * c, wlr_scale + 2 * c);
  const float *fold = lnproj ? ln_w : nullptr;
  if (!pw.fresh) {
    // prepared by an earlier call with these weights
  } else if (!L.split) {
    const PrepJob jobs[3] = {
        {left_m, cm, c, L.cmp, c, 1.f, wp + L.off_wlr, wlr_scale, 0, lr_cols, fold},
        {right_m, cm, c, L.cmp, c, 1.f, wp + L.off_wlr, wlr_scale, c, lr_cols, fold},
        {out_m, c * c, cz, o_inner, o_cols, std::ldexp(1.f, L.out_shift), wp + L.off_wo, wo_scale, 0, 0}};
    if ((st = prepare_matrices(ctx, jobs, 3, stream)) != AF2_OK) return st;
  } else {
    // K-tripled weights [W_hi; W_lo; W_hi] against the operands [hi | hi | lo] (norm and outer kernels)
    const int part[3] = {0, 1, 0};
    PrepJob lr[6], wo[3];
    for (int g = 0; g < 3; ++g) {
      uint8_t *seg = wp + L.off_wlr + (size_t)g * L.cmp * lr_cols * 2;
      lr[2 * g] = PrepJob{left_m, cm, c, L.cmp, c, 1.f, seg, wlr_scale, 0, lr_cols, nullptr, part[g]};
      lr[2 * g + 1] = PrepJob{right_m, cm, c, L.cmp, c, 1.f, seg, wlr_scale, c, lr_cols, nullptr, part[g]};
      wo[g] = PrepJob{out_m, c * c, cz, o_inner, o_cols, std::ldexp(1.f, L.out_shift),
                      wp + L.off_wo + (size_t)g * o_inner * o_cols * 2, wo_scale, 0, 0, nullptr, part[g]};
    }
    if ((st = prepare_matrices(ctx, lr, 6, stream)) != AF2_OK || (st = prepare_matrices(ctx, wo, 3, stream)) != AF2_OK)
      return st;
  }
  if (pw.fresh && (st = pad_vectors(ctx, vs, stream)) != AF2_OK) return st;
  if (lnproj && pw.fresh) {
    LaunchScope scope(ctx, stream, kProfPrepare);
    fold_beta_kernel<<<(unsigned)((2 * c + 7) / 8), 256, 0, stream>>>(ln_b, lw, rw, (int)cm, (int)c, wlr_bias);
    if (cudaError_t e = cudaGetLastError(); e != cudaSuccess) return cuda_fail(ctx, e, "OPM LayerNorm fold");
  }
  __half *right_full = reinterpret_cast<__half *>(ws + L.off_right);
  if (lnproj) {
    CUtensorMap mmap;
    // m [S][m_cols][c_m] viewed as {c_m, m_cols, S}: a box is 64 channels x 1 residue x 128 sequences
    if (!encode_map_3d(&mmap, m_dtype == AF2_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                       m, cm, m_cols, s, cm * 2, (uint64_t)m_cols * cm * 2, 64, 1, 128, CU_TENSOR_MAP_SWIZZLE_128B))
      return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the OPM's MSA map");
    LnProjArgs a{};
    a.scale = wlr_scale;
    a.bias = wlr_bias;
    a.mask = mask;
    a.w = reinterpret_cast<const __half *>(wp + L.off_wlr);
    a.left = reinterpret_cast<__half *>(ws + L.off_left);
    a.right = right_full + (size_t)rank * L.seq_pitch * rows * c;
    a.n_full = n;
    a.m_row0 = (int)m_col0;
    a.rows = rows;
    a.pitch = L.seq_pitch;
    a.row0 = (int)L.row0;
    a.s_count = (int)s;
    a.cm = (int)cm;
    a.chunks = (int)(L.cmp / 64);
    a.n_sb = (int)((s + 127) / 128);
    a.total_tiles = (int)(rows * a.n_sb);
    a.eps = (float)ln_eps;
    a.err = ctx->err_word;
    const int grid = std::max(1, std::min(a.total_tiles, ctx->sm_count));
    auto run = [&](auto tag) -> cudaError_t {
      using MT = decltype(tag);
      cudaError_t e = cudaFuncSetAttribute(lnproj_kernel<MT>, cudaFuncAttributeMaxDynamicSharedMemorySize, LP_SMEM);
      if (e != cudaSuccess) return e;
      LaunchScope scope(ctx, stream, kProfOpmProject);
      lnproj_kernel<MT><<<grid, LP_THREADS, LP_SMEM, stream>>>(mmap, a);
      return cudaGetLastError();
    };
    const cudaError_t e = m_dtype == AF2_BF16 ? run(__nv_bfloat16{}) : run(__half{});
    if (e != cudaSuccess) return cuda_fail(ctx, e, "OPM LayerNorm and projection");
  }
  // ---- LayerNorm of this rank's residue columns (all of them unless sharded) ----
  const int64_t xrows = s * rows;
  __half *xn = reinterpret_cast<__half *>(ws + L.off_xn);
  float *mask_loc = reinterpret_cast<float *>(ws + L.off_mask);
  if (!lnproj) {
    const int warps = 8;
    const unsigned blocks = (unsigned)((xrows + warps - 1) / warps);
    LaunchScope scope(ctx, stream, kProfOpmNormalize);
    const bool vec = cm == 256 && reinterpret_cast<uintptr_t>(m) % 16 == 0;
    auto run = [&](auto tag) {
      using MT = decltype(tag);
      const MT *mp = static_cast<const MT *>(m);
      if (vec)
        norm_kernel<MT, true><<<blocks, warps * 32, 0, stream>>>(mp, xrows, (int)cm, (int)L.cmp, ln, ln + L.cmp,
                                                                 (float)ln_eps, xn, (int)n, (int)L.row0, (int)rows,
                                                                 L.fused ? (int)s : 0, mask, mask_loc, L.split, (int)m_cols, (int)m_col0);
      else
        norm_kernel<MT, false><<<blocks, warps * 32, 0, stream>>>(mp, xrows, (int)cm, (int)L.cmp, ln, ln + L.cmp,
                                                                  (float)ln_eps, xn, (int)n, (int)L.row0, (int)rows,
                                                                  L.fused ? (int)s : 0, mask, mask_loc, L.split, (int)m_cols, (int)m_col0);
    };
    if (m_dtype == AF2_F32)
      run(float{});
    else if (m_dtype == AF2_F16)
      run(__half{});
    else
      run(__nv_bfloat16{});
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "OPM normalisation");
  }
  // ---- left / right projection: right lands in this rank's block of the full operand ----
  if (!lnproj) {
    LinearOperands op;
    op.a = xn;
    op.lda = kx * L.cmp;
    op.inner = kx * L.cmp;
    op.w = wp + L.off_wlr;
    if (L.split) {
      op.split_stride_left = s * rows * c;
      op.split_stride_right = s * n * c;
    }
    op.scale = wlr_scale;
    op.bias = wlr_bias;
    op.row_mask = mask_loc;
    op.rows = xrows;
    op.cols = 2 * c;
    op.opm_projection = true;
    op.left = ws + L.off_left;
    op.kmajor_rows = rows;
    op.kmajor_seqs = s;
    op.seq_pitch = L.seq_pitch;
    op.right = right_full + (size_t)rank * (L.fused ? L.seq_pitch : s) * rows * c;
    op.prof = kProfOpmProject;
    if ((st = linear_launch(ctx, op, stream)) != AF2_OK) return st;
  }
  if (exchange && exchange->all_gather &&
      (st = exchange->all_gather(ctx, right_full, (size_t)(L.fused ? L.seq_pitch : s) * rows * c * sizeof(__half),
                                 stream)) != AF2_OK)
    return st;
  // ---- pair counts of this rank's rows ----
  float *rowscale = reinterpret_cast<float *>(ws + L.off_rowscale);
  {
    LaunchScope scope(ctx, stream, kProfOpmCount);
    const dim3 grid((unsigned)((n + CNT_TILE - 1) / CNT_TILE), (unsigned)((rows + CNT_TILE - 1) / CNT_TILE));
    count_kernel<<<grid, CNT_THREADS, 0, stream>>>(mask, (int)s, (int)n, (int)L.row0, (int)rows, (float)norm_eps,
                                                   rowscale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "OPM pair counts");
  }
  if (L.fused) return fused_launch(ctx, L, ws, wp, right_full, residual, out, out_dtype, stream);
  const int64_t blocks_b = n / rows;  // blocks of the right operand
  // ---- outer products and output projection, block by block of this rank's rows ----
  CUtensorMap lmap, rmap;
  // the split operands are three stacked [S][rows][c] blocks: one contraction over 3 S sequences
  const int64_t sk = kx * s;
  if (!encode_map_3d(&lmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_left, rows * c, sk, 1, rows * c * 2,
                     (uint64_t)sk * rows * c * 2, 64, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&rmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, right_full, rows * c, sk, blocks_b, rows * c * 2,
                     (uint64_t)sk * rows * c * 2, 64, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the OPM operands");
  cudaError_t e = cudaFuncSetAttribute(outer_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, OSMEM);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "outer kernel attributes");
  __half *outer = reinterpret_cast<__half *>(ws + L.off_outer);
  const size_t ob_bytes = out_dtype == AF2_F32 ? 4 : 2;
  for (int64_t i0 = 0; i0 < rows; i0 += L.block_rows) {
    const int64_t ic = std::min<int64_t>(L.block_rows, rows - i0);
    OuterArgs a{};
    a.outer = outer;
    a.n = (int)n;
    a.i_begin = (int)i0;
    a.i_count = (int)ic;
    a.tiles_j = (int)((n + 7) / 8);
    a.k_blocks = (int)((sk + OBK - 1) / OBK);
    a.split = L.split ? 1 : 0;
    a.total_tiles = (int)((ic + 3) / 4) * a.tiles_j;
    a.rows_b = (int)rows;
    a.scale = std::ldexp(1.f, -L.out_shift);
    a.err = ctx->err_word;
    {
      LaunchScope scope(ctx, stream, kProfOpmOuter);
      outer_kernel<<<std::min(a.total_tiles, ctx->sm_count), OTHREADS, OSMEM, stream>>>(lmap, rmap, a);
      e = cudaGetLastError();
      if (e != cudaSuccess) return cuda_fail(ctx, e, "outer kernel launch");
    }
    LinearOperands op;
    op.a = outer;
    op.lda = kx * c * c;
    op.inner = kx * c * c;
    op.w = wp + L.off_wo;
    op.scale = wo_scale;
    op.bias = wo_bias;
    op.row_scale = rowscale + i0 * n;
    op.rows = ic * n;
    op.cols = cz;
    op.out = static_cast<uint8_t *>(out) + (size_t)i0 * n * cz * ob_bytes;
    op.ldo = cz;
    op.out_dtype = out_dtype;
    op.residual = residual;
    op.prof = kProfOpmOutput;
    if ((st = linear_launch(ctx, op, stream)) != AF2_OK) return st;
  }
  return AF2_OK;
}

}  // namespace af2
