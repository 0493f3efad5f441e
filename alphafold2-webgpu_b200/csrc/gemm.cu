// gemm.cu -- the shared dense projection on sm_100a: weight preparation (f32
// or mixed-q8 [in, out] matrices -> f16 operand rows with per-column scales)
// and one persistent tcgen05 GEMM, D = A W, with the epilogues its callers
// need: the linear layer out (=, +=) act(scale * D + bias) (optionally times a
// per-row factor), and the outer-product-mean projection that splits the
// masked result into its left and right operands.
//
// Reference: src/evoformer/transition.ts:91-138 (createLinearShader: A W + b,
// optional ReLU, optional accumulate into the output) and
// src/runtime/gemm.ts:836-1000 (the tiled GEMM it is written against);
// src/evoformer/outer-product-mean.ts:189-231 (the masked left/right
// projection) and :433-486 (the output projection, divided per pair by
// norm_eps + count).
//
// Kernel: one CTA per SM, 128-row tiles of A times BN-column tiles of W (BN
// <= 256), K in 64-wide blocks through a 4-deep TMA ring; warp 0 issues TMA,
// warp 1 the tcgen05 MMAs into one of two TMEM accumulators, warps 2-9 drain
// the other accumulator (one TMEM lane = one output row per thread; two warps
// per lane quarter, taking alternate 32-column chunks).
#include <algorithm>
#include <cstring>
#include <type_traits>
#include <string>

#include "af2_device.cuh"
#include "af2_internal.h"

namespace af2 {
namespace gemm {

constexpr int BM = 128, BK = 64, STAGES = 4;
constexpr int EPI_WARPS = 8;  // two per TMEM lane quarter
constexpr int THREADS = 64 + 32 * EPI_WARPS;
constexpr uint32_t A_BYTES = BM * 128;

struct LinearArgs {
  const float *scale, *bias;  // per output column (padded to the tile)
  const float *row_scale;     // per output row, or NULL
  const float *row_mask;      // OPM projection: mask per row
  void *out;                  // LINEAR: [rows][ldo] of OT
  __half *left, *right;       // OPM projection: [rows][half_cols] each
  int64_t split_left, split_right;  // OPM projection, f32 mode: element distance of the split blocks (0: off)
  int64_t kmajor_rows, kmajor_seqs, seq_pitch;  // seq_pitch > 0: rows m = i * seqs + s, outputs sequence-contiguous
  int64_t rows, ldo;
  int cols, half_cols, k_blocks, tiles_m, tiles_n, total_tiles, bn;
  int relu, residual;
  int vector_out;  // out rows are 16-byte aligned: whole 32-column chunks use vector access
  int tma_out;     // f16 output, no residual: each warp stages 32 x 32 blocks and stores them by TMA
  int stage_bufs;  // staging blocks per epilogue warp (2 when shared memory allows: a store in flight
                   // while the next block is staged)
  // LINEAR: with transpose_q > 0 row m = b * transpose_q + q is written to row q * transpose_b + b
  // (the attention output of a transposed view goes back to its source row)
  int64_t transpose_q, transpose_b;
  // ATTENTION projection: columns [q | k | v | g | bias] of width C, C, C, C, heads; rows m = b * queries + j
  __half *att_q, *att_k, *att_vt, *att_g, *att_bias;
  int64_t att_queries, att_pitch;  // key pitch of the transposed values and of the bias rows
  int att_c, att_heads;
  unsigned int *err;
};

// Per epilogue warp: one 32-row x 32-column f16 staging block for the TMA-stored output.
constexpr uint32_t OUT_STAGE_BYTES = 32 * 64;
// The column scales and biases, copied to shared memory once per CTA when there are at most this
// many columns (the epilogue reads 64 of them per 32-column chunk; from global memory each read
// goes to L2, since the operand ring leaves L1 little room).
constexpr int kSmemVecCols = 1024;
constexpr uint32_t VEC_BYTES = 2 * kSmemVecCols * 4;

enum { kModeLinear = 0, kModeOpmProjection = 1, kModeAttentionProjection = 2 };

// Attention projection: TMA store maps of q and k ([b][h][j][32], boxes 32 x 32 rows) and of the
// transposed values ([b][h][32 d][j], boxes 32 keys x 32 d); the gate goes through `omap`.
struct AttentionMaps {
  CUtensorMap q, k, v;
};

template <typename OT, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    linear_kernel(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap,
                  const __grid_constant__ CUtensorMap omap, const __grid_constant__ AttentionMaps amaps,
                  const LinearArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t B_BYTES = p.bn * 128u, STAGE_BYTES = A_BYTES + B_BYTES;
  const uint32_t OFF_BAR = STAGES * STAGE_BYTES;
  const uint32_t bar0 = sbase + OFF_BAR;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  auto acc_full = [&](int b) { return bar0 + 8u * (2 * STAGES + b); };
  auto acc_empty = [&](int b) { return bar0 + 8u * (2 * STAGES + 2 + b); };
  const uint32_t drain = bar0 + 8u * (2 * STAGES + 4);
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_BAR + 128);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + 136);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(acc_full(b), 1);
      mbar_init(acc_empty(b), EPI_WARPS);
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
    // ---- TMA producer ----
    if (lane == 0) {
      tma_prefetch_map(&amap);
      tma_prefetch_map(&bmap);
      int it = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x) {
        const int mi = t / p.tiles_n, ni = t - mi * p.tiles_n;
        for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t dst = sbase + s * STAGE_BYTES;
          mbar_arrive_expect_tx(full(s), STAGE_BYTES);
          tma_load_3d(dst, &amap, full(s), kb * BK, mi * BM, 0);
          tma_load_3d(dst + A_BYTES, &bmap, full(s), 0, ni * p.bn, kb);
        }
      }
      for (int j = std::max(0, it - STAGES); j < it; ++j) mbar_wait_drain(full(j % STAGES), (j / STAGES) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_f16_f32(BM, p.bn);
    const uint64_t a_desc = sdesc_k_sw128(sbase);
    int it = 0, tile_it = 0;
    bool ok = true;
    for (int t = blockIdx.x; ok && t < p.total_tiles; t += gridDim.x, ++tile_it) {
      const int buf = tile_it & 1;
      if (!warp_wait(acc_empty(buf), ((tile_it >> 1) & 1) ^ 1, abort_flag, p.err, kErrWaitMma)) break;
      tc_fence_after();
      const uint32_t d = tmem + buf * 256;
      for (int kb = 0; kb < p.k_blocks; ++kb, ++it) {
        const int s = it % STAGES;
        if (!warp_wait(full(s), (it / STAGES) & 1, abort_flag, p.err, kErrWaitMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint64_t ad = desc_add(a_desc, s * STAGE_BYTES), bd = desc_add(ad, A_BYTES);
        if (kb == 0)
          umma_first(d, ad, bd, idesc);
        else
          umma_acc(d, ad, bd, idesc);
#pragma unroll
        for (int ks = 1; ks < BK / 16; ++ks) umma_acc(d, desc_add(ad, ks * 32), desc_add(bd, ks * 32), idesc);
        umma_commit(empty(s));
      }
      if (ok) umma_commit(acc_full(buf));
    }
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else {
    // ---- epilogue: one output row per thread, alternate column chunks per warp of a quarter ----
    const int q = warp & 3, half = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    // the staged path exists for f16 outputs only (the host sets tma_out accordingly)
    const bool staged = MODE == kModeLinear && std::is_same<OT, __half>::value && p.tma_out;
    const uint32_t stage_base = OFF_BAR + 256 + (warp - 2) * p.stage_bufs * OUT_STAGE_BYTES;
    int sb = 0;  // the staging block this warp fills next
    const int cols_pad = p.tiles_n * p.bn;
    const float *vscale = p.scale, *vbias = p.bias;
    if (cols_pad <= kSmemVecCols) {
      float *sv = reinterpret_cast<float *>(smem + OFF_BAR + 256 + EPI_WARPS * p.stage_bufs * OUT_STAGE_BYTES);
      for (int i = threadIdx.x - 64; i < cols_pad; i += 32 * EPI_WARPS) {
        sv[i] = p.scale[i];
        sv[kSmemVecCols + i] = p.bias[i];
      }
      named_barrier(1, 32 * EPI_WARPS);  // the epilogue warps only
      vscale = sv;
      vbias = sv + kSmemVecCols;
    }
    bool store_pending = false;
    int tile_it = 0;
    for (int t = blockIdx.x; t < p.total_tiles; t += gridDim.x, ++tile_it) {
      const int mi = t / p.tiles_n, ni = t - mi * p.tiles_n;
      const int buf = tile_it & 1;
      if (!warp_wait(acc_full(buf), (tile_it >> 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      const int64_t m = static_cast<int64_t>(mi) * BM + row;
      const bool row_ok = m < p.rows;
      const int n0 = ni * p.bn;
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + buf * 256;
      float rs = 1.f;
      if (MODE == kModeLinear && p.row_scale && row_ok) rs = p.row_scale[m];
      // LINEAR with a transposed view: the row of the source this output row belongs to
      int64_t m_out = m;
      if (MODE == kModeLinear && p.transpose_q > 0) {
        const int64_t tb = m / p.transpose_q;
        m_out = (m - tb * p.transpose_q) * p.transpose_b + tb;
      }
      if (MODE == kModeOpmProjection && row_ok) rs = p.row_mask[m];
      for (int chunk = half; chunk < p.bn / 32; chunk += 2) {
        uint32_t v[32];
        tmem_ld32(taddr + chunk * 32, v);
        tmem_ld_wait();
        const int c0 = n0 + chunk * 32;
        if (staged) {
          // rows past p.rows and columns past p.cols are staged too and the TMA store drops them;
          // a block that starts past the last row or column is not stored at all
          if (c0 >= p.cols || static_cast<int64_t>(mi) * BM + q * 32 >= p.rows) continue;
          uint32_t pk[16];
          const float4 *sc = reinterpret_cast<const float4 *>(vscale + c0);
          const float4 *bi = reinterpret_cast<const float4 *>(vbias + c0);
#pragma unroll
          for (int i4 = 0; i4 < 8; ++i4) {
            const float4 s4 = sc[i4], b4 = bi[i4];
            float y0 = fmaf(__uint_as_float(v[4 * i4 + 0]), s4.x, b4.x) * rs;
            float y1 = fmaf(__uint_as_float(v[4 * i4 + 1]), s4.y, b4.y) * rs;
            float y2 = fmaf(__uint_as_float(v[4 * i4 + 2]), s4.z, b4.z) * rs;
            float y3 = fmaf(__uint_as_float(v[4 * i4 + 3]), s4.w, b4.w) * rs;
            if (p.relu) {
              y0 = fmaxf(y0, 0.f), y1 = fmaxf(y1, 0.f), y2 = fmaxf(y2, 0.f), y3 = fmaxf(y3, 0.f);
            }
            pk[2 * i4] = pack_half2(y0, y1);
            pk[2 * i4 + 1] = pack_half2(y2, y3);
          }
          // the store that last used this block has read it
          if (lane == 0 && store_pending) {
            if (p.stage_bufs > 1)
              bulk_wait_read_but_one();
            else
              bulk_wait_read_all();
          }
          __syncwarp();
          const uint32_t stage_off = stage_base + sb * OUT_STAGE_BYTES;
          sb = sb + 1 == p.stage_bufs ? 0 : sb + 1;
          // row `lane` of the block is 64 bytes; its four 16-byte pieces are written in an order
          // rotated by the lane, so each store instruction covers every bank once per 128 bytes
          uint8_t *stage_row = smem + stage_off + lane * 64;
          const uint4 q0 = make_uint4(pk[0], pk[1], pk[2], pk[3]), q1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
          const uint4 q2 = make_uint4(pk[8], pk[9], pk[10], pk[11]), q3 = make_uint4(pk[12], pk[13], pk[14], pk[15]);
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int pc = (w + lane) & 3;
            *reinterpret_cast<uint4 *>(stage_row + pc * 16) = pc == 0 ? q0 : pc == 1 ? q1 : pc == 2 ? q2 : q3;
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_3d(&omap, sbase + stage_off, c0, mi * BM + q * 32, 0);
            bulk_commit();
            store_pending = true;
          }
          continue;
        }
        if (MODE == kModeAttentionProjection) {
          // a 32-row block inside one batch row b0 (and, for the values, starting on a 16-byte
          // boundary) leaves through shared memory and one TMA store: q, k, gate as rows of 64
          // bytes, the values transposed as 32 d rows of 32 keys
          const int C = p.att_c, part = c0 / C, cc = c0 - part * C, h = cc >> 5;
          const int64_t m0 = static_cast<int64_t>(mi) * BM + q * 32;
          const int64_t b0 = m0 / p.att_queries, j0 = m0 - b0 * p.att_queries;
          if (part <= 3 && m0 < p.rows && j0 + 32 <= p.att_queries && (part != 2 || j0 % 8 == 0)) {
            float y[32];
            const float4 *sc = reinterpret_cast<const float4 *>(vscale + c0);
            const float4 *bi = reinterpret_cast<const float4 *>(vbias + c0);
#pragma unroll
            for (int i4 = 0; i4 < 8; ++i4) {
              const float4 s4 = sc[i4], b4 = bi[i4];
              y[4 * i4 + 0] = fmaf(__uint_as_float(v[4 * i4 + 0]), s4.x, b4.x);
              y[4 * i4 + 1] = fmaf(__uint_as_float(v[4 * i4 + 1]), s4.y, b4.y);
              y[4 * i4 + 2] = fmaf(__uint_as_float(v[4 * i4 + 2]), s4.z, b4.z);
              y[4 * i4 + 3] = fmaf(__uint_as_float(v[4 * i4 + 3]), s4.w, b4.w);
            }
            // the store that last used this block has read it
            if (lane == 0 && store_pending) {
              if (p.stage_bufs > 1)
                bulk_wait_read_but_one();
              else
                bulk_wait_read_all();
            }
            __syncwarp();
            const uint32_t stage_off = stage_base + sb * OUT_STAGE_BYTES;
            sb = sb + 1 == p.stage_bufs ? 0 : sb + 1;
            if (part == 2) {
              __half *st = reinterpret_cast<__half *>(smem + stage_off);
#pragma unroll
              for (int d = 0; d < 32; ++d) st[d * 32 + lane] = __float2half_rn(y[d]);
            } else {
              uint32_t pk[16];
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                float y0 = y[2 * i], y1 = y[2 * i + 1];
                if (part == 3) y0 = sigmoidf(y0), y1 = sigmoidf(y1);
                pk[i] = pack_half2(y0, y1);
              }
              uint8_t *stage_row = smem + stage_off + lane * 64;
              const uint4 q0 = make_uint4(pk[0], pk[1], pk[2], pk[3]), q1 = make_uint4(pk[4], pk[5], pk[6], pk[7]);
              const uint4 q2 = make_uint4(pk[8], pk[9], pk[10], pk[11]),
                          q3 = make_uint4(pk[12], pk[13], pk[14], pk[15]);
#pragma unroll
              for (int w = 0; w < 4; ++w) {
                const int pc = (w + lane) & 3;
                *reinterpret_cast<uint4 *>(stage_row + pc * 16) = pc == 0 ? q0 : pc == 1 ? q1 : pc == 2 ? q2 : q3;
              }
            }
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
              const uint32_t src = sbase + stage_off;
              if (part == 0)
                tma_store_4d(&amaps.q, src, 0, (int)j0, h, (int)b0);
              else if (part == 1)
                tma_store_4d(&amaps.k, src, 0, (int)j0, h, (int)b0);
              else if (part == 2)
                tma_store_4d(&amaps.v, src, (int)j0, 0, h, (int)b0);
              else
                tma_store_3d(&omap, src, cc, (int)m0, 0);
              bulk_commit();
              store_pending = true;
            }
            continue;
          }
        }
        if (!row_ok || c0 >= p.cols) continue;
        float y[32];
        const float4 *sc = reinterpret_cast<const float4 *>(vscale + c0);
        const float4 *bi = reinterpret_cast<const float4 *>(vbias + c0);
#pragma unroll
        for (int i4 = 0; i4 < 8; ++i4) {
          const float4 s4 = sc[i4], b4 = bi[i4];
          y[4 * i4 + 0] = fmaf(__uint_as_float(v[4 * i4 + 0]), s4.x, b4.x);
          y[4 * i4 + 1] = fmaf(__uint_as_float(v[4 * i4 + 1]), s4.y, b4.y);
          y[4 * i4 + 2] = fmaf(__uint_as_float(v[4 * i4 + 2]), s4.z, b4.z);
          y[4 * i4 + 3] = fmaf(__uint_as_float(v[4 * i4 + 3]), s4.w, b4.w);
        }
        if (MODE == kModeAttentionProjection) {
          // gated attention projections of row m = (b, j) (src/evoformer/attention.ts:497-566 and the
          // pair-bias projection :631-661): q, k -> [b][h][j][32]; v -> transposed [b][h][32][j];
          // g = sigmoid(.) -> [m][C]; bias[h][q = b][k = j] -> transposed [h][j][b].  The scales carry log2(e) / sqrt(d) for q
          // and log2(e) for the bias, so the flash kernel works in base 2.
          const int C = p.att_c, part = c0 / C, cc = c0 - part * C, h = cc >> 5;
          const int64_t b = m / p.att_queries, j = m - b * p.att_queries;
          const int64_t bh = b * p.att_heads + h;
          if (part <= 1 || part == 3) {
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              float y0 = y[2 * i], y1 = y[2 * i + 1];
              if (part == 3) y0 = sigmoidf(y0), y1 = sigmoidf(y1);
              pk[i] = pack_half2(y0, y1);
            }
            __half *dst = part == 0   ? p.att_q + (bh * p.att_queries + j) * 32
                          : part == 1 ? p.att_k + (bh * p.att_queries + j) * 32
                                      : p.att_g + m * C + cc;
            uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
            for (int w = 0; w < 4; ++w) d4[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
          } else if (part == 2) {
            // the lanes of a warp hold consecutive keys j: each store covers 64 contiguous bytes
            __half *dst = p.att_vt + bh * 32 * p.att_pitch + j;
#pragma unroll
            for (int d = 0; d < 32; ++d) dst[d * p.att_pitch] = __float2half_rn(y[d]);
          } else if (part == 4 && cc == 0 && p.att_bias) {
            // bias[h][q = b][k = j], stored transposed as [h][k][q] (rows of queries)
            for (int hh = 0; hh < p.att_heads; ++hh)
              p.att_bias[(static_cast<int64_t>(hh) * p.att_queries + j) * p.att_pitch + b] = __float2half_rn(y[hh]);
          }
          continue;
        }
        if (MODE == kModeOpmProjection) {
          // columns [0, half) -> left, [half, 2 half) -> right, both scaled by the mask;
          // half is 32, so a chunk is one whole left or right row: 4 x 16-byte stores.
          if (p.seq_pitch) {
            // K-major operands of the outer products, sequences contiguous: row m = (i, s) ->
            // left[a][i][s], right[i][b][s], one channel per store; the lanes of a warp hold
            // consecutive sequences, so a store covers 64 contiguous bytes
            const int64_t i = m / p.kmajor_seqs, sq = m - i * p.kmajor_seqs;
            const bool is_left = c0 < p.half_cols;
            __half *dst = is_left ? p.left + i * p.seq_pitch + sq : p.right + i * p.half_cols * p.seq_pitch + sq;
            const int64_t stride = is_left ? p.kmajor_rows * p.seq_pitch : p.seq_pitch;
#pragma unroll
            for (int k = 0; k < 32; ++k) dst[k * stride] = __float2half_rn(y[k] * rs);
            continue;
          }
          const bool is_left = c0 < p.half_cols;
          __half *dst = (is_left ? p.left : p.right) + m * p.half_cols;
          uint32_t pk[16];
          if (p.split_left) {
            // f32 precision mode: hi = f16(v), lo = f16(v - hi); left blocks (hi, hi, lo), right (hi, lo, hi)
            uint32_t lo[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float v0 = y[2 * i] * rs, v1 = y[2 * i + 1] * rs;
              const __half h0 = __float2half_rn(v0), h1 = __float2half_rn(v1);
              pk[i] = pack_half2(__half2float(h0), __half2float(h1));
              lo[i] = pack_half2(v0 - __half2float(h0), v1 - __half2float(h1));
            }
            const int64_t stride = is_left ? p.split_left : p.split_right;
            uint4 *b0 = reinterpret_cast<uint4 *>(dst), *b1 = reinterpret_cast<uint4 *>(dst + stride),
                  *b2 = reinterpret_cast<uint4 *>(dst + 2 * stride);
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const uint4 hv = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
              const uint4 lv = make_uint4(lo[4 * w], lo[4 * w + 1], lo[4 * w + 2], lo[4 * w + 3]);
              b0[w] = hv;
              b1[w] = is_left ? hv : lv;
              b2[w] = is_left ? lv : hv;
            }
            continue;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack_half2(y[2 * i] * rs, y[2 * i + 1] * rs);
          uint4 *d4 = reinterpret_cast<uint4 *>(dst);
#pragma unroll
          for (int w = 0; w < 4; ++w) d4[w] = make_uint4(pk[4 * w], pk[4 * w + 1], pk[4 * w + 2], pk[4 * w + 3]);
        } else {
          OT *orow = static_cast<OT *>(p.out) + m_out * p.ldo;
#pragma unroll
          for (int i = 0; i < 32; ++i) y[i] = (p.relu ? fmaxf(y[i], 0.f) : y[i]) * rs;
          store_out32<OT>(orow, c0, p.cols, y, p.vector_out, p.residual);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(acc_empty(buf));
    }
    if (lane == 0 && store_pending) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// Weight preparation: an [inner][cols] matrix (f32, q8 block or q8 channel)
// -> f16 operand rows [inner_pad / 64][cols_pad][64] (K-blocked, one row per
// output column) and a per-column f32 scale.  For q8 channel weights the rows
// hold the int8 codes (exact in f16) and the scale is the given one; for f32
// and q8 block weights (decoded exactly to f32 first) the scale is the power
// of two bringing the column's largest magnitude into [0.5, 1).
// ---------------------------------------------------------------------------
constexpr int PREP_THREADS = 256;
constexpr int PREP_CHUNK = 128;  // K rows converted per CTA

struct MatrixDev {
  int format, block;
  const void *values, *scales;
};

template <int FMT>
__device__ __forceinline__ float element(const MatrixDev &m, int64_t i) {
  if (FMT == AF2_WEIGHTS_F32) return static_cast<const float *>(m.values)[i];
  const float code = static_cast<float>(static_cast<const int8_t *>(m.values)[i]);
  if (FMT == AF2_WEIGHTS_Q8_CHANNEL) return code;
  const uint16_t bits = static_cast<const uint16_t *>(m.scales)[i / m.block];
  return code * __half2float(__ushort_as_half(bits));
}

struct PrepJobDev {
  MatrixDev m;
  int inner, cols, inner_pad, cols_pad, row0, rows_total, part;
  float extra_scale;
  __half *out;
  float *scale_out;
  const float *row_scale;  // NULL, or a factor per inner row k
};
struct PrepBatch {
  PrepJobDev job[kMaxPrepJobs];
};

// CTA (column group of 32, chunk of 128 K rows, job).  The column's scale
// needs the maximum over all of its K rows: every CTA of the column group
// takes it (a read that stays in L2), so no CTA waits for another; the chunk
// 0 CTA stores the scales.  Then the chunk is rounded to f16 and written as
// rows [k / 64][rows_total][64] (one 128-byte row segment per column and K block).
template <int FMT>
__device__ __forceinline__ void prep_chunk(const PrepJobDev &jb) {
  __shared__ float red[PREP_THREADS / 32][33];
  __shared__ float col_scale[32];
  __shared__ __align__(16) __half stage[32][PREP_CHUNK + 8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int o0 = blockIdx.x * 32, o = o0 + lane;
  const int k0 = blockIdx.y * PREP_CHUNK;
  if (o0 >= jb.cols_pad || k0 >= jb.inner_pad) return;
  constexpr bool codes = FMT == AF2_WEIGHTS_Q8_CHANNEL;
  if (!codes) {
    float mx = 0.f;
    if (o < jb.cols)
      for (int k = warp; k < jb.inner; k += PREP_THREADS / 32)
        mx = fmaxf(mx, fabsf(element<FMT>(jb.m, static_cast<int64_t>(k) * jb.cols + o) *
                             (jb.row_scale ? jb.row_scale[k] : 1.f)));
    red[warp][lane] = mx;
  }
  __syncthreads();
  if (warp == 0) {
    float scale = 1.f;
    if (o < jb.cols) {
      if (codes) {
        scale = static_cast<const float *>(jb.m.scales)[o];
      } else {
        float v = 0.f;
        for (int w = 0; w < PREP_THREADS / 32; ++w) v = fmaxf(v, red[w][lane]);
        if (v > 0.f && isfinite(v)) {
          int e;
          frexpf(v, &e);
          scale = ldexpf(1.f, e);
        }
      }
    }
    col_scale[lane] = scale;
    if (blockIdx.y == 0 && o < jb.cols_pad) jb.scale_out[jb.row0 + o] = scale * jb.extra_scale;
  }
  __syncthreads();
  const float inv = codes ? 1.f : 1.f / col_scale[lane];
  const int kend = min(k0 + PREP_CHUNK, jb.inner_pad);
  for (int k = k0 + warp; k < kend; k += PREP_THREADS / 32) {
    float w = 0.f;
    if (o < jb.cols && k < jb.inner)
      w = element<FMT>(jb.m, static_cast<int64_t>(k) * jb.cols + o) * (jb.row_scale ? jb.row_scale[k] : 1.f) * inv;
    const __half hw = __float2half_rn(w);
    stage[lane][k - k0] = jb.part ? __float2half_rn(w - __half2float(hw)) : hw;
  }
  __syncthreads();
  const int kblocks = (kend - k0) >> 6;  // inner_pad is a multiple of 64
  for (int i = threadIdx.x; i < kblocks * 256; i += PREP_THREADS) {
    const int blk = i >> 8, r = (i >> 3) & 31, c16 = i & 7;
    if (o0 + r < jb.cols_pad) {
      const uint4 v = *reinterpret_cast<const uint4 *>(&stage[r][blk * 64 + c16 * 8]);
      *reinterpret_cast<uint4 *>(
          jb.out + ((static_cast<int64_t>((k0 >> 6) + blk) * jb.rows_total + jb.row0 + o0 + r) * 64 + c16 * 8)) = v;
    }
  }
}

__global__ void __launch_bounds__(PREP_THREADS) prep_matrix_kernel(const PrepBatch batch) {
  const PrepJobDev &jb = batch.job[blockIdx.z];
  if (jb.m.format == AF2_WEIGHTS_Q8_CHANNEL)
    prep_chunk<AF2_WEIGHTS_Q8_CHANNEL>(jb);
  else if (jb.m.format == AF2_WEIGHTS_Q8_BLOCK)
    prep_chunk<AF2_WEIGHTS_Q8_BLOCK>(jb);
  else
    prep_chunk<AF2_WEIGHTS_F32>(jb);
}

// Segment k: dst[i] = i < n ? src[i] : 0 for i < n_pad (src may be NULL: zeros).
__global__ void pad_vectors_kernel(VectorSegments v) {
  const int k = blockIdx.y;
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (k < v.count && i < v.n_pad[k]) v.dst[k][i] = (v.src[k] && i < v.n[k]) ? v.src[k][i] : 0.f;
}

// f32 / 16-bit rows [rows][inner] -> f16 rows [rows][inner_pad] (zero padded).
template <typename T>
__global__ void to_f16_kernel(const T *__restrict__ src, int64_t rows, int inner, int inner_pad,
                              __half *__restrict__ dst) {
  const int64_t total = rows * inner_pad;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / inner_pad;
    const int k = static_cast<int>(i - r * inner_pad);
    dst[i] = __float2half_rn(k < inner ? to_f32<T>(src[r * inner + k]) : 0.f);
  }
}

}  // namespace gemm

using namespace gemm;

namespace {
CUtensorMapDataType f16map() { return CU_TENSOR_MAP_DATA_TYPE_FLOAT16; }
}  // namespace

af2_status prepare_matrices(af2_ctx *ctx, const PrepJob *jobs, int count, cudaStream_t stream) {
  if (count < 1 || count > kMaxPrepJobs) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "weight preparation batch size");
  PrepBatch b{};
  unsigned gx = 1, gy = 1;
  for (int i = 0; i < count; ++i) {
    const PrepJob &j = jobs[i];
    b.job[i] = PrepJobDev{MatrixDev{j.w.format, j.w.block, j.w.values, j.w.scales},
                          (int)j.inner, (int)j.cols, (int)j.inner_pad, (int)j.cols_pad, (int)j.row0,
                          (int)(j.rows_total ? j.rows_total : j.cols_pad), j.part, j.extra_scale,
                          static_cast<__half *>(j.out), j.scale_out, j.row_scale};
    gx = std::max(gx, (unsigned)((j.cols_pad + 31) / 32));
    gy = std::max(gy, (unsigned)((j.inner_pad + PREP_CHUNK - 1) / PREP_CHUNK));
  }
  LaunchScope scope(ctx, stream, kProfPrepare);
  prep_matrix_kernel<<<dim3(gx, gy, (unsigned)count), PREP_THREADS, 0, stream>>>(b);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "weight preparation");
}

af2_status prepare_matrix(af2_ctx *ctx, const af2_matrix &w, int64_t inner, int64_t cols, int64_t inner_pad,
                          int64_t cols_pad, float extra_scale, void *out, float *scale_out, cudaStream_t stream,
                          int64_t row0, int64_t rows_total) {
  const PrepJob job{w, inner, cols, inner_pad, cols_pad, extra_scale, out, scale_out, row0, rows_total};
  return prepare_matrices(ctx, &job, 1, stream);
}

af2_status pad_vectors(af2_ctx *ctx, const VectorSegments &v, cudaStream_t stream) {
  int widest = 1;
  for (int k = 0; k < v.count; ++k) widest = std::max(widest, v.n_pad[k]);
  LaunchScope scope(ctx, stream, kProfPrepare);
  pad_vectors_kernel<<<dim3((unsigned)((widest + 255) / 256), (unsigned)v.count), 256, 0, stream>>>(v);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "vector preparation");
}

af2_status pad_vector(af2_ctx *ctx, const float *src, int64_t n, int64_t n_pad, float *dst, cudaStream_t stream) {
  VectorSegments v{};
  v.add(src, n, n_pad, dst);
  return pad_vectors(ctx, v, stream);
}

af2_status convert_rows_f16(af2_ctx *ctx, const void *src, int dtype, int64_t rows, int64_t inner, int64_t inner_pad,
                            void *dst, cudaStream_t stream) {
  const int threads = 256;
  const unsigned blocks = (unsigned)std::min<int64_t>((rows * inner_pad + threads - 1) / threads, 8LL * ctx->sm_count * 8);
  LaunchScope scope(ctx, stream, kProfConvert);
  __half *d = static_cast<__half *>(dst);
  if (dtype == AF2_F32)
    to_f16_kernel<float><<<blocks, threads, 0, stream>>>(static_cast<const float *>(src), rows, (int)inner,
                                                         (int)inner_pad, d);
  else if (dtype == AF2_BF16)
    to_f16_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(static_cast<const __nv_bfloat16 *>(src), rows,
                                                                 (int)inner, (int)inner_pad, d);
  else
    to_f16_kernel<__half><<<blocks, threads, 0, stream>>>(static_cast<const __half *>(src), rows, (int)inner,
                                                          (int)inner_pad, d);
  cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "activation conversion");
}

namespace {

template <typename OT, int MODE>
af2_status launch_linear_t(af2_ctx *ctx, const CUtensorMap &amap, const CUtensorMap &bmap, const CUtensorMap &omap,
                           const AttentionMaps &amaps, const LinearArgs &a, int prof, cudaStream_t stream) {
  auto kernel = linear_kernel<OT, MODE>;
  const uint32_t smem =
      STAGES * (A_BYTES + a.bn * 128u) + 256 + EPI_WARPS * a.stage_bufs * OUT_STAGE_BYTES + VEC_BYTES + 1024;
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return cuda_fail(ctx, e, "linear kernel attributes");
  const int grid = std::min(a.total_tiles, ctx->sm_count);
  LaunchScope scope(ctx, stream, prof);
  kernel<<<grid, THREADS, smem, stream>>>(amap, bmap, omap, amaps, a);
  e = cudaGetLastError();
  return e == cudaSuccess ? AF2_OK : cuda_fail(ctx, e, "linear kernel launch");
}

}  // namespace

af2_status linear_launch(af2_ctx *ctx, const LinearOperands &op, cudaStream_t stream) {
  const int64_t k_pad = align_up(op.inner, 64);
  const int bn = op.bn > 0 ? op.bn : op.cols >= 256 ? 256 : (int)align_up(op.cols, 64);
  const int64_t cols_pad = align_up(op.cols, bn);
  CUtensorMap amap, bmap;
  // A: f16 rows of pitch lda; K past `inner` reads as zero (TMA fill), matching the zero-padded W rows.
  if (!encode_map_3d(&amap, f16map(), op.a, op.inner, op.rows, 1, op.lda * 2, (uint64_t)op.rows * op.lda * 2, 64, BM, 1,
                     CU_TENSOR_MAP_SWIZZLE_128B) ||
      !encode_map_3d(&bmap, f16map(), op.w, 64, cols_pad, k_pad / 64, 128, (uint64_t)cols_pad * 128, 64, bn, 1,
                     CU_TENSOR_MAP_SWIZZLE_128B))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for a linear layer");
  LinearArgs a{};
  a.scale = op.scale;
  a.bias = op.bias;
  a.row_scale = op.row_scale;
  a.row_mask = op.row_mask;
  a.out = op.out;
  a.left = static_cast<__half *>(op.left);
  a.right = static_cast<__half *>(op.right);
  a.split_left = op.split_stride_left;
  a.split_right = op.split_stride_right;
  a.kmajor_rows = op.kmajor_rows;
  a.kmajor_seqs = op.kmajor_seqs;
  a.seq_pitch = op.seq_pitch;
  a.rows = op.rows;
  a.ldo = op.ldo;
  a.cols = (int)op.cols;
  a.half_cols = (int)(op.cols / 2);
  a.k_blocks = (int)(k_pad / 64);
  a.tiles_m = (int)((op.rows + BM - 1) / BM);
  a.tiles_n = (int)(cols_pad / bn);
  a.total_tiles = a.tiles_m * a.tiles_n;
  a.bn = bn;
  a.relu = op.relu;
  a.residual = op.residual;
  a.transpose_q = op.transpose_q;
  a.transpose_b = op.transpose_b;
  const bool attention = op.attention != nullptr;
  if (attention) {
    a.att_q = static_cast<__half *>(op.attention->q);
    a.att_k = static_cast<__half *>(op.attention->k);
    a.att_vt = static_cast<__half *>(op.attention->vt);
    a.att_g = static_cast<__half *>(op.attention->g);
    a.att_bias = static_cast<__half *>(op.attention->bias);
    a.att_queries = op.attention->queries;
    a.att_pitch = op.attention->pitch;
    a.att_c = (int)op.attention->channels;
    a.att_heads = (int)op.attention->heads;
  }
  {
    const size_t ob = op.out_dtype == AF2_F32 ? 4 : 2;
    a.vector_out = !op.opm_projection && reinterpret_cast<uintptr_t>(op.out) % 16 == 0 && (op.ldo * ob) % 16 == 0;
  }
  a.err = ctx->err_word;
  // f16 outputs without a residual leave through staged TMA stores: [rows][ldo], one box = 32 x 32
  CUtensorMap omap;
  std::memset(&omap, 0, sizeof omap);
  a.tma_out = !op.opm_projection && !attention && op.out_dtype == AF2_F16 && !op.residual && a.vector_out &&
              op.transpose_q == 0;
  if (a.tma_out && !encode_map_3d(&omap, f16map(), op.out, op.cols, op.rows, 1, op.ldo * 2,
                                  (uint64_t)op.rows * op.ldo * 2, 32, 32, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
    return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for a linear layer's output");
  // two staging blocks per epilogue warp where shared memory holds them (tiles up to 192 columns)
  a.stage_bufs = STAGES * (A_BYTES + a.bn * 128u) + 256 + EPI_WARPS * 2 * OUT_STAGE_BYTES + VEC_BYTES + 1024 <= 232448u
                     ? 2
                     : 1;
  AttentionMaps amaps;
  std::memset(&amaps, 0, sizeof amaps);
  if (attention) {
    const AttentionProjection &ap = *op.attention;
    const int64_t B = op.rows / ap.queries, Q = ap.queries, H = ap.heads;
    const uint64_t qk_dims[4] = {32, (uint64_t)Q, (uint64_t)H, (uint64_t)B};
    const uint64_t qk_strides[3] = {64, (uint64_t)Q * 64, (uint64_t)H * Q * 64};
    const uint32_t qk_box[4] = {32, 32, 1, 1};
    const uint64_t v_dims[4] = {(uint64_t)Q, 32, (uint64_t)H, (uint64_t)B};
    const uint64_t v_strides[3] = {(uint64_t)ap.pitch * 2, (uint64_t)32 * ap.pitch * 2, (uint64_t)H * 32 * ap.pitch * 2};
    const uint32_t v_box[4] = {32, 32, 1, 1};
    if (!encode_map_4d(&amaps.q, f16map(), ap.q, qk_dims, qk_strides, qk_box, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_map_4d(&amaps.k, f16map(), ap.k, qk_dims, qk_strides, qk_box, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_map_4d(&amaps.v, f16map(), ap.vt, v_dims, v_strides, v_box, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !encode_map_3d(&omap, f16map(), ap.g, ap.channels, op.rows, 1, ap.channels * 2,
                       (uint64_t)op.rows * ap.channels * 2, 32, 32, 1, CU_TENSOR_MAP_SWIZZLE_NONE))
      return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the attention projection's outputs");
  }
  if (op.opm_projection)
    return launch_linear_t<__half, kModeOpmProjection>(ctx, amap, bmap, omap, amaps, a, op.prof, stream);
  if (attention)
    return launch_linear_t<__half, kModeAttentionProjection>(ctx, amap, bmap, omap, amaps, a, op.prof, stream);
  if (op.out_dtype == AF2_F16)
    return launch_linear_t<__half, kModeLinear>(ctx, amap, bmap, omap, amaps, a, op.prof, stream);
  if (op.out_dtype == AF2_BF16)
    return launch_linear_t<__nv_bfloat16, kModeLinear>(ctx, amap, bmap, omap, amaps, a, op.prof, stream);
  return launch_linear_t<float, kModeLinear>(ctx, amap, bmap, omap, amaps, a, op.prof, stream);
}

}  // namespace af2

namespace af2 {

// Scratch of af2_linear: prepared weights, their column scales and biases,
// and an f16 copy of A when A is not already f16 rows with a 16-byte pitch.
LinearLayout linear_layout(int64_t rows, int64_t inner, int64_t cols, int a_dtype) {
  LinearLayout L;
  L.k_pad = align_up(inner, 64);
  L.cols_pad = linear_cols_pad(cols);
  L.convert = a_dtype != AF2_F16 || inner % 8 != 0;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.off_w = take((size_t)L.k_pad * L.cols_pad * 2);
  L.off_scale = take((size_t)L.cols_pad * 4);
  L.off_bias = take((size_t)L.cols_pad * 4);
  L.off_a = L.convert ? take((size_t)rows * L.k_pad * 2) : off;
  L.total = off;
  return L;
}

af2_status linear_run(af2_ctx *ctx, const LinearLayout &L, int64_t rows, int64_t inner, int64_t cols, const void *a,
                      int a_dtype, const af2_matrix &weight, const float *bias, int activation, int residual,
                      void *out, int out_dtype, void *workspace, cudaStream_t stream) {
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  // the prepared weights: the layout's prefix [0, off_a), in the weight cache or the workspace
  WeightKey key;
  key.kind = kWeightsLinear;
  key.ptr[0] = weight.values;
  key.ptr[1] = weight.scales;
  key.ptr[2] = bias;
  key.dim[0] = inner;
  key.dim[1] = cols;
  key.dim[2] = weight.format * 65536 + weight.block;
  PreparedRegion pw;
  af2_status st = prepared_region(ctx, key, L.off_a, ws, true, &pw);
  if (st != AF2_OK) return st;
  uint8_t *wp = pw.base;
  float *scale = reinterpret_cast<float *>(wp + L.off_scale), *bvec = reinterpret_cast<float *>(wp + L.off_bias);
  if (pw.fresh &&
      ((st = prepare_matrix(ctx, weight, inner, cols, L.k_pad, L.cols_pad, 1.f, wp + L.off_w, scale, stream)) !=
           AF2_OK ||
       (st = pad_vector(ctx, bias, bias ? cols : 0, L.cols_pad, bvec, stream)) != AF2_OK))
    return st;
  LinearOperands op;
  op.a = a;
  op.lda = inner;
  if (L.convert) {
    if ((st = convert_rows_f16(ctx, a, a_dtype, rows, inner, L.k_pad, ws + L.off_a, stream)) != AF2_OK) return st;
    op.a = ws + L.off_a;
    op.lda = L.k_pad;
  }
  op.inner = inner;
  op.w = wp + L.off_w;
  op.scale = scale;
  op.bias = bvec;
  op.rows = rows;
  op.cols = cols;
  op.out = out;
  op.ldo = cols;
  op.out_dtype = out_dtype;
  op.relu = activation == AF2_ACTIVATION_RELU;
  op.residual = residual;
  op.prof = kProfLinear;
  return linear_launch(ctx, op, stream);
}

}  // namespace af2
