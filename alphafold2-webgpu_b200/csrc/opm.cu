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
//   normalize  LayerNorm of every MSA row -> f16 [S*N][c_m]
//   project    the shared tcgen05 GEMM: LN(m) [W_left | W_right], bias, times
//              the row's mask, split into left and right, f16 [S][N][c]
//   count      1 / (norm_eps + sum_s mask[s,i] mask[s,j]) per pair
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
                            int cols, const float *__restrict__ mask_in, float *__restrict__ mask_out) {
  // local row (s, j) of the residue columns [col0, col0 + cols) of an [S][n_full] MSA
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t src = (row / cols) * n_full + col0 + row % cols;
  if (lane == 0) mask_out[row] = mask_in[src];
  const MT *xr = m + src * cm;
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
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      pk[i] = pack_half2((v[2 * i] - mean) * rstd * g[2 * i] + b[2 * i],
                         (v[2 * i + 1] - mean) * rstd * g[2 * i + 1] + b[2 * i + 1]);
    reinterpret_cast<uint4 *>(xn + row * cmp)[lane] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int ch = lane + 32 * i;
      if (ch < cmp)
        xn[row * cmp + ch] = __float2half_rn(ch < cm ? (v[i] - mean) * rstd * gamma[ch] + beta[ch] : 0.f);
    }
  }
}

// ---- pair counts: rowscale[i*N + j] = 1 / (norm_eps + sum_s mask[s,i] mask[s,j]) ----
// A 32 x 32 block of pairs per CTA; 64 MSA rows of both residue columns at a
// time through shared memory; every count sums s in order.
__global__ void __launch_bounds__(256) count_kernel(const float *__restrict__ mask, int s_count, int n, int row0,
                                                    int rows, float norm_eps, float *__restrict__ rowscale) {
  // rows i in [row0, row0 + rows), stored from row 0 of rowscale
  __shared__ float mi[64][33], mj[64][33];
  const int i0 = row0 + blockIdx.y * 32, j0 = blockIdx.x * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int s0 = 0; s0 < s_count; s0 += 64) {
    for (int r = ty; r < 64; r += 8) {
      const int64_t s = s0 + r;
      mi[r][tx] = (s < s_count && i0 + tx < row0 + rows) ? mask[s * n + i0 + tx] : 0.f;
      mj[r][tx] = (s < s_count && j0 + tx < n) ? mask[s * n + j0 + tx] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int r = 0; r < 64; ++r) {
      const float b = mj[r][tx];
#pragma unroll
      for (int k = 0; k < 4; ++k) acc[k] = fmaf(mi[r][ty + 8 * k], b, acc[k]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int i = i0 + ty + 8 * k, j = j0 + tx;
    if (i < row0 + rows && j < n) rowscale[static_cast<int64_t>(i - row0) * n + j] = 1.f / (norm_eps + acc[k]);
  }
}

// ---- outer products: outer[(i, j)][a*32 + b] = 2^-shift sum_s left[s][i][a] right[s][j][b] ----
constexpr int OBM = 128, OBN = 256, OBK = 64, OSTAGES = 4, OTHREADS = 192;
constexpr uint32_t OA_BYTES = OBM * 128, OB_BYTES = OBN * 128, OSTAGE = OA_BYTES + OB_BYTES;
constexpr uint32_t OOFF_BAR = OSTAGES * OSTAGE;
constexpr uint32_t OSMEM = OOFF_BAR + 256 + 1024;

struct OuterArgs {
  __half *outer;  // [(i - i_begin) * n + j][1024]
  int n, i_begin, i_count, tiles_j, k_blocks, total_tiles;
  int rows_b;     // residues per block of the right operand ([blocks][S][rows_b][c]): n unless sharded
  float scale;
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
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

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
    if (lane == 0) {
      // both operands MN-major: 64-element MN blocks 8 KB apart, 8-row K groups 1 KB apart
      constexpr uint32_t kIdesc = idesc_f16_f32(OBM, OBN) | (1u << 15) | (1u << 16);
      const uint64_t a_desc = sdesc_mn_sw128(sbase, 8192, 1024);
      int it = 0, tile_it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x, ++tile_it) {
        const int buf = tile_it & 1;
        if (!mbar_wait(acc_empty(buf), ((tile_it >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitMma)) break;
        tc_fence_after();
        const uint32_t d = tmem + buf * OBN;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % OSTAGES;
          if (!mbar_wait(full(s), (it / OSTAGES) & 1, abort_flag, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = desc_add(a_desc, s * OSTAGE), bd = desc_add(ad, OA_BYTES);
          if (kb == 0)
            mma_f16_first(d, ad, bd, kIdesc);
          else
            mma_f16_acc(d, ad, bd, kIdesc);
#pragma unroll
          for (int ks = 1; ks < OBK / 16; ++ks) mma_f16_acc(d, desc_add(ad, ks * 2048), desc_add(bd, ks * 2048), kIdesc);
          mma_commit(empty(s));
        }
        if (ok) mma_commit(acc_full(buf));
      }
      mma_commit(drain);
      mbar_wait_drain(drain, 0, p.err);
    }
    __syncwarp();
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
        uint4 *dst = reinterpret_cast<uint4 *>(p.outer + (static_cast<int64_t>(i - p.i_begin) * p.n + j) * (C * C) +
                                              lane * C);
#pragma unroll
        for (int w = 0; w < 4; ++w) dst[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
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

}  // namespace opm

using namespace opm;

OpmLayout opm_layout(int64_t s, int64_t n, int64_t cm, int64_t c, int64_t cz, int64_t row_block, int64_t rows,
                     int64_t row0) {
  OpmLayout L;
  L.s = s;
  L.n = n;
  L.rows = (rows <= 0 || rows > n) ? n : rows;
  L.row0 = row0;
  L.cm = cm;
  L.c = c;
  L.cz = cz;
  L.cmp = align_up(cm, 64);
  // Residue block: the outer scratch stays within 256 MiB unless asked otherwise; a multiple of 4.
  int64_t rb = row_block > 0 ? row_block : std::max<int64_t>(4, (int64_t(256) << 20) / (n * c * c * 2));
  rb = std::min<int64_t>(align_up(std::max<int64_t>(rb, 1), 4), align_up(L.rows, 4));
  L.block_rows = rb;
  int k = 0;
  while ((int64_t(1) << k) < s) ++k;
  L.out_shift = k;
  const int64_t lr_cols = linear_cols_pad(2 * c), o_cols = linear_cols_pad(cz), o_inner = align_up(c * c, 64);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.off_wlr = take((size_t)L.cmp * lr_cols * 2);
  L.off_wlr_scale = take((size_t)lr_cols * 4);
  L.off_wlr_bias = take((size_t)lr_cols * 4);
  L.off_wo = take((size_t)o_inner * o_cols * 2);
  L.off_wo_scale = take((size_t)o_cols * 4);
  L.off_wo_bias = take((size_t)o_cols * 4);
  L.off_ln = take((size_t)L.cmp * 2 * 4);
  L.off_xn = take((size_t)s * L.rows * L.cmp * 2);
  L.off_mask = take((size_t)s * L.rows * 4);
  L.off_left = take((size_t)s * L.rows * c * 2);
  L.off_right = take((size_t)s * n * c * 2);  // every rank's block [ranks][S][rows][c]
  L.off_rowscale = take((size_t)L.rows * n * 4);
  L.off_outer = take((size_t)rb * n * c * c * 2);
  L.total = off;
  return L;
}

af2_status opm_launch(af2_ctx *ctx, const OpmLayout &L, const void *m, int m_dtype, const float *mask,
                      const float *packed, double ln_eps, double norm_eps, int residual, void *out, int out_dtype,
                      void *workspace, cudaStream_t stream, const OpmExchange *exchange) {
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int64_t s = L.s, n = L.n, cm = L.cm, c = L.c, cz = L.cz, rows = L.rows;
  const int rank = exchange ? exchange->rank : 0;
  // packOuterProductMeanWeights order (outer-product-mean.ts:68-72).
  const float *ln_w = packed, *ln_b = ln_w + cm, *lw = ln_b + cm, *lb = lw + cm * c, *rw = lb + c, *rb = rw + cm * c;
  const float *ow = rb + c, *ob = ow + c * c * cz;
  const int64_t lr_cols = linear_cols_pad(2 * c), o_cols = linear_cols_pad(cz), o_inner = align_up(c * c, 64);
  float *wlr_scale = reinterpret_cast<float *>(ws + L.off_wlr_scale), *wlr_bias = reinterpret_cast<float *>(ws + L.off_wlr_bias);
  float *wo_scale = reinterpret_cast<float *>(ws + L.off_wo_scale), *wo_bias = reinterpret_cast<float *>(ws + L.off_wo_bias);
  float *ln = reinterpret_cast<float *>(ws + L.off_ln);
  af2_status st;
  // ---- weights ----
  const af2_matrix left_m{AF2_WEIGHTS_F32, 0, lw, nullptr}, right_m{AF2_WEIGHTS_F32, 0, rw, nullptr};
  const af2_matrix out_m{AF2_WEIGHTS_F32, 0, ow, nullptr};
  VectorSegments vs{};
  vs.add(lb, c, c, wlr_bias);
  vs.add(rb, c, lr_cols - c, wlr_bias + c);
  vs.add(ob, cz, o_cols, wo_bias);
  vs.add(ln_w, cm, L.cmp, ln);
  vs.add(ln_b, cm, L.cmp, ln + L.cmp);
  if (lr_cols > 2 * c) vs.add(nullptr, 0, lr_cols - 2 * c, wlr_scale + 2 * c);
  if ((st = prepare_matrix(ctx, left_m, cm, c, L.cmp, c, 1.f, ws + L.off_wlr, wlr_scale, stream, 0, lr_cols)) != AF2_OK ||
      (st = prepare_matrix(ctx, right_m, cm, c, L.cmp, c, 1.f, ws + L.off_wlr, wlr_scale, stream, c, lr_cols)) !=
          AF2_OK ||
      (st = prepare_matrix(ctx, out_m, c * c, cz, o_inner, o_cols, std::ldexp(1.f, L.out_shift), ws + L.off_wo,
                           wo_scale, stream)) != AF2_OK ||
      (st = pad_vectors(ctx, vs, stream)) != AF2_OK)
    return st;
  // ---- LayerNorm of this rank's residue columns (all of them unless sharded) ----
  const int64_t xrows = s * rows;
  __half *xn = reinterpret_cast<__half *>(ws + L.off_xn);
  float *mask_loc = reinterpret_cast<float *>(ws + L.off_mask);
  {
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
                                                                 mask, mask_loc);
      else
        norm_kernel<MT, false><<<blocks, warps * 32, 0, stream>>>(mp, xrows, (int)cm, (int)L.cmp, ln, ln + L.cmp,
                                                                  (float)ln_eps, xn, (int)n, (int)L.row0, (int)rows,
                                                                  mask, mask_loc);
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
  __half *right_full = reinterpret_cast<__half *>(ws + L.off_right);
  {
    LinearOperands op;
    op.a = xn;
    op.lda = L.cmp;
    op.inner = L.cmp;
    op.w = ws + L.off_wlr;
    op.scale = wlr_scale;
    op.bias = wlr_bias;
    op.row_mask = mask_loc;
    op.rows = xrows;
    op.cols = 2 * c;
    op.opm_projection = true;
    op.left = ws + L.off_left;
    op.right = right_full + (size_t)rank * s * rows * c;
    op.prof = kProfOpmProject;
    if ((st = linear_launch(ctx, op, stream)) != AF2_OK) return st;
  }
  if (exchange && exchange->all_gather &&
      (st = exchange->all_gather(ctx, right_full, (size_t)s * rows * c * sizeof(__half), stream)) != AF2_OK)
    return st;
  // ---- pair counts of this rank's rows ----
  float *rowscale = reinterpret_cast<float *>(ws + L.off_rowscale);
  {
    LaunchScope scope(ctx, stream, kProfOpmCount);
    const dim3 grid((unsigned)((n + 31) / 32), (unsigned)((rows + 31) / 32));
    count_kernel<<<grid, 256, 0, stream>>>(mask, (int)s, (int)n, (int)L.row0, (int)rows, (float)norm_eps, rowscale);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "OPM pair counts");
  }
  // ---- outer products and output projection, block by block of this rank's rows ----
  const int64_t blocks_b = n / rows;  // blocks of the right operand
  CUtensorMap lmap, rmap;
  if (!encode_map_3d(&lmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_left, rows * c, s, 1, rows * c * 2,
                     (uint64_t)s * rows * c * 2, 64, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&rmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, right_full, rows * c, s, blocks_b, rows * c * 2,
                     (uint64_t)s * rows * c * 2, 64, 64, 1, CU_TENSOR_MAP_SWIZZLE_128B))
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
    a.k_blocks = (int)((s + OBK - 1) / OBK);
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
    op.lda = c * c;
    op.inner = c * c;
    op.w = ws + L.off_wo;
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
