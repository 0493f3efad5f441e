// attention.cu -- gated multi-head attention on sm_100a, as the Evoformer's
// triangle attention runs it: the pair [N, N, C] attends along each row
// (starting node) or, through the transposed view, along each column (ending
// node), with a per-head bias projected from the same normalised pair.
//
// Reference: AttentionGpu.run and encodeAttention (src/evoformer/attention.ts:
// 1321-1453; the in-model calls src/evoformer/block.ts:1727-1745): LayerNorm
// of the source rows (:243-336), the q / k / v / gate projections (:497-566),
// the pair bias bias[h][q][k] = LN(x)[q, k] . W_b[:, h] (:631-661), the flash
// loop logit = q.k / sqrt(d) + 1e9 (mask[k] - 1) + bias, clamped to +-1e8,
// softmax over the keys, times the gate (ATTENTION_FLASH_SHADER :663-731),
// and the output projection written back to the source row (:1261-1314).
//
// Kernels (one call):
//   attn_norm_kernel    LayerNorm of every source row (the transposed view reads
//                       the pair column-wise), f16 rows [B*Q][C];
//   attn_mask_kernel    the additive key mask 1e9 (mask - 1), in base 2, [B][Q];
//   linear_kernel       (gemm.cu, attention epilogue) one tcgen05 GEMM of the
//                       normalised rows by [Wq | Wk | Wv | Wg | Wb]: q (times
//                       log2(e)/sqrt(d)) and k as [b][h][j][32], v transposed
//                       as [b][h][32][j], sigmoid(gate) as [b*Q + j][C], the
//                       pair bias (times log2(e)) transposed, [h][k][q];
//   attn_flash_kernel   the flash loop, below;
//   linear_kernel       the output projection, added into the pair rows.
//
// The flash kernel (one CTA per SM, persistent): a unit of work is one head h,
// a pair of batch rows (b0, b1) and a block of 128 queries.  Two softmax
// warpgroups own one batch row each and share the bias tile of (h, query
// block, key block), which both rows read (the bias does not depend on the
// batch row).  Per block of 128 keys: warp 0 loads by TMA both rows' K (128 x
// 32) and transposed V (32 x 128), the bias tile (128 x 128, f16) and both
// rows' key masks into a 3-stage ring; warp 1 issues S_g = Q_g K_g^T (M 128,
// N 128, K 32) into TMEM, then, once group g has written P_g (f16) into TMEM,
// O_g += P_g V_g (M 128, N 32, K 128, A read from TMEM); each softmax thread
// owns one query row (one TMEM lane): it reads its S row, adds bias and mask,
// clamps, keeps the running maximum and sum in base 2, rescales its O row when
// the maximum grows, and writes P.  After the last key block it divides O by
// the sum, multiplies by the gate and writes the weighted values (f16) for the
// output projection.  S of the next key block is computed while the softmax of
// this one runs.
#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <type_traits>

#include "af2_device.cuh"
#include "af2_internal.h"

namespace af2 {
namespace attn {

constexpr float kLog2e = 1.4426950408889634f;
// 1e8 in base-2 logit units: the reference clamps logits to +-1e8 before the softmax
constexpr float kClamp = 1.0e8f * 1.4426950408889634f;

// ---- LayerNorm of the source rows ------------------------------------------
// Row m = b * Q + q of the view is source row m (transpose = 0) or q * B + b
// (transpose = 1: the column view, AttentionInput.transpose).  One warp per
// row; C is a multiple of 32 (head dimension 32), at most 256.
template <typename T>
__global__ void attn_norm_kernel(const T *__restrict__ x, int64_t rows, int C, int64_t B, int64_t Q, int transpose,
                                 const float *__restrict__ gamma, const float *__restrict__ beta, float eps,
                                 __half *__restrict__ xn) {
  const int lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (m >= rows) return;
  const int64_t b = m / Q, q = m - b * Q;
  const int64_t src = transpose ? q * B + b : m;
  const T *row = x + src * C;
  const int per = C >> 5;
  float v[8];
  float sum = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[i] = i < per ? to_f32<T>(row[lane + 32 * i]) : 0.f;
    sum += v[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
  const float mean = sum / static_cast<float>(C);
  float var = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) {
      const float c = v[i] - mean;
      var += c * c;
    }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(kFull, var, o);
  const float inv = rsqrtf(var / static_cast<float>(C) + eps);
  __half *out = xn + m * C;
#pragma unroll
  for (int i = 0; i < 8; ++i)
    if (i < per) {
      const int c = lane + 32 * i;
      out[c] = __float2half_rn((v[i] - mean) * inv * gamma[c] + beta[c]);
    }
}

// The same LayerNorm for C = 128, four rows per warp: lane l holds channels 4l .. 4l + 3 of each
// row (one 8-byte load of a 16-bit row, 16 bytes of an f32 one), the four rows' loads issued
// together; two-pass statistics over the row held in registers, as above.
template <typename T>
__global__ void attn_norm128_kernel(const T *__restrict__ x, int64_t rows, int64_t B, int64_t Q, int transpose,
                                    const float *__restrict__ gamma, const float *__restrict__ beta, float eps,
                                    __half *__restrict__ xn) {
  constexpr int R = 4;
  const int lane = threadIdx.x & 31;
  const int64_t m0 = (static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5)) * R;
  if (m0 >= rows) return;
  float v[R][4];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t m = m0 + r;
    if (m < rows) {
      const int64_t b = m / Q, q = m - b * Q;
      const T *row = x + (transpose ? q * B + b : m) * 128 + 4 * lane;
      if constexpr (std::is_same<T, float>::value) {
        const float4 f = *reinterpret_cast<const float4 *>(row);
        v[r][0] = f.x, v[r][1] = f.y, v[r][2] = f.z, v[r][3] = f.w;
      } else {
        const uint2 u = *reinterpret_cast<const uint2 *>(row);
        const float2 a = unpack2<T>(u.x), c = unpack2<T>(u.y);
        v[r][0] = a.x, v[r][1] = a.y, v[r][2] = c.x, v[r][3] = c.y;
      }
    } else {
      v[r][0] = v[r][1] = v[r][2] = v[r][3] = 0.f;
    }
  }
  const float4 g = reinterpret_cast<const float4 *>(gamma)[lane], bt = reinterpret_cast<const float4 *>(beta)[lane];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float sum = (v[r][0] + v[r][1]) + (v[r][2] + v[r][3]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(kFull, sum, o);
    const float mean = sum * (1.f / 128.f);
    const float c0 = v[r][0] - mean, c1 = v[r][1] - mean, c2 = v[r][2] - mean, c3 = v[r][3] - mean;
    float var = (c0 * c0 + c1 * c1) + (c2 * c2 + c3 * c3);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(kFull, var, o);
    const float inv = rsqrtf(var * (1.f / 128.f) + eps);
    if (m0 + r < rows) {
      const uint2 o = make_uint2(pack_half2(c0 * inv * g.x + bt.x, c1 * inv * g.y + bt.y),
                                 pack_half2(c2 * inv * g.z + bt.z, c3 * inv * g.w + bt.w));
      *reinterpret_cast<uint2 *>(xn + (m0 + r) * 128 + 4 * lane) = o;
    }
  }
}

// mb[b][k] = 1e9 (mask - 1) log2(e) for the view's row b and key k (mask_index, attention.ts:428-433).
__global__ void attn_mask_kernel(const float *__restrict__ mask, int64_t B, int64_t Q, int transpose, int64_t pitch,
                                 float *__restrict__ mb) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= B * Q) return;
  const int64_t b = i / Q, k = i - b * Q;
  const float mv = mask[transpose ? k * B + b : i];
  mb[b * pitch + k] = (mv - 1.f) * 1.0e9f * kLog2e;
}

// ---- the flash kernel --------------------------------------------------------

constexpr int THREADS = 320;  // warp 0 TMA, warp 1 MMA, warps 2-9 softmax (two groups of four)
constexpr int STAGES = 3;
constexpr uint32_t K_BYTES = 128 * 64;         // [128 keys][32 d] f16, 64B-swizzled
constexpr uint32_t V_BYTES = 32 * 128 * 2;     // [32 d][128 keys] f16 as two 64-key boxes, 128B-swizzled
constexpr uint32_t BIAS_BYTES = 128 * 128 * 2; // [128 keys][128 q] f16 as two 64-query boxes
constexpr uint32_t MB_BYTES = 128 * 4;
constexpr uint32_t OFF_K = 0, OFF_V = 2 * K_BYTES, OFF_BIAS = OFF_V + 2 * V_BYTES, OFF_MB = OFF_BIAS + BIAS_BYTES;
constexpr uint32_t STAGE_BYTES = OFF_MB + 2 * MB_BYTES;  // 66,560: a multiple of 1024
constexpr uint32_t Q_BYTES = 128 * 64;
constexpr uint32_t OFF_Q = STAGES * STAGE_BYTES;
constexpr uint32_t OFF_BAR = OFF_Q + 2 * Q_BYTES;
constexpr uint32_t SMEM_BYTES = OFF_BAR + 256 + 1024;
static_assert(STAGE_BYTES % 1024 == 0, "stages keep the 1024-byte swizzle alignment");
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");

// TMEM columns of softmax group g: S at 256 g, P (f16 pairs) at 256 g + 128, O at 256 g + 192
// (to 256 g + 224).  The identity A operand that adds the bias tile to S on the tensor core
// (shared by both groups) fills the two 32-column gaps: K steps 0-3 (queries 0-63) at 224,
// K steps 4-7 (queries 64-127) at 480.
constexpr uint32_t TM_GROUP = 256, TM_P = 128, TM_O = 192, TM_I0 = 224, TM_I1 = 480;
__host__ __device__ constexpr uint32_t tm_identity(int ks) { return (ks < 4 ? TM_I0 : TM_I1) + 8u * (ks & 3); }
// The running maximum moves only when a row's maximum grows by more than this (base 2): the
// probabilities stay below 2^8, exact enough in f16, and O is rescaled far less often.
constexpr float kLazyRescale = 8.f;

struct FlashArgs {
  __half *weighted;        // [B * Q][C]
  const __half *gate;      // [B * Q][C]
  const int *flags;        // [B][nkb]: the key block has masked keys or keys past Q
  int64_t batch, queries;
  int channels, heads, nqb, nkb, nbp, units, has_bias;
  unsigned int *err;
};

__device__ __forceinline__ float ex2f(float v) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(v));
  return r;
}

// flags[b][kb] = 1 when block kb of row b has a key with mask != 1 or runs past the last key:
// only those blocks take the mask add and the clamp (one warp per block).
__global__ void attn_flag_kernel(const float *__restrict__ mask, int64_t B, int64_t Q, int transpose, int nkb,
                                 int *__restrict__ flags) {
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (w >= B * nkb) return;
  const int64_t b = w / nkb, k0 = (w - b * nkb) * 128;
  bool any = false;
  for (int i = lane; i < 128; i += 32) {
    const int64_t k = k0 + i;
    any |= k >= Q || mask[transpose ? k * B + b : b * Q + k] != 1.f;
  }
  any = __any_sync(kFull, any);
  if (lane == 0) flags[w] = any ? 1 : 0;
}

// Ten warps put three on two of the four SM sub-partitions, whose 16,384 registers then cap a
// thread at 168.
__global__ void __launch_bounds__(THREADS, 1)
    attn_flash_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const __grid_constant__ CUtensorMap bmap,
                      const __grid_constant__ CUtensorMap mmap, const FlashArgs p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t *smem = align1024(smem_raw);
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + OFF_BAR;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (STAGES + s); };
  const uint32_t q_full = bar0 + 8u * (2 * STAGES), q_empty = q_full + 8u;
  auto s_full = [&](int g) { return q_full + 16u + 8u * g; };
  auto s_free = [&](int g) { return q_full + 32u + 8u * g; };
  auto p_full = [&](int g) { return q_full + 48u + 8u * g; };
  auto o_done = [&](int g) { return q_full + 64u + 8u * g; };
  const uint32_t drain = q_full + 80u;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(smem + OFF_BAR + 192);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + OFF_BAR + 200);
  const int warp = warp_index_uniform(), lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1 + 8);  // the MMAs that read the stage, and the eight softmax warps (mask)
    }
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int g = 0; g < 2; ++g) {
      mbar_init(s_full(g), 1);
      mbar_init(s_free(g), 4);
      mbar_init(p_full(g), 4);
      mbar_init(o_done(g), 1);
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
  if (warp >= 2 && warp < 6) {
    // the 128 x 128 identity, f16 pairs along K: lane r holds 1.0 at column r
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>((warp & 3) * 32) << 16;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const uint32_t taddr = tmem + lanes + (half ? TM_I1 : TM_I0);
      uint32_t v[32];
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int col = 32 * half + c;
        v[c] = (r == 2 * col) ? 0x00003C00u : (r == 2 * col + 1) ? 0x3C000000u : 0u;
      }
      tmem_st32(taddr, v);
    }
    tmem_st_wait();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const int nkb = p.nkb;
  const uint32_t stage_tx = 2 * K_BYTES + 2 * V_BYTES + (p.has_bias ? BIAS_BYTES : 0) + 2 * MB_BYTES;

  if (warp == 0) {
    // ---- TMA producer ----
    if (lane == 0) {
      tma_prefetch_map(&qmap);
      tma_prefetch_map(&kmap);
      tma_prefetch_map(&vmap);
      if (p.has_bias) tma_prefetch_map(&bmap);
      tma_prefetch_map(&mmap);
      int it = 0, uit = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++uit) {
        const int qb = u % p.nqb, rest = u / p.nqb, bp = rest % p.nbp, h = rest / p.nbp;
        if (!mbar_wait(q_empty, (uit & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) break;
        mbar_arrive_expect_tx(q_full, 2 * Q_BYTES);
        for (int g = 0; g < 2; ++g)
          tma_load_4d(sbase + OFF_Q + g * Q_BYTES, &qmap, q_full, 0, qb * 128, h, 2 * bp + g);
        for (int kb = 0; kb < nkb; ++kb, ++it) {
          const int s = it % STAGES;
          if (!mbar_wait(empty(s), ((it / STAGES) & 1) ^ 1, abort_flag, p.err, kErrWaitProducer)) {
            ok = false;
            break;
          }
          const uint32_t st = sbase + s * STAGE_BYTES;
          mbar_arrive_expect_tx(full(s), stage_tx);
          for (int g = 0; g < 2; ++g) {
            const int b = 2 * bp + g;
            tma_load_4d(st + OFF_K + g * K_BYTES, &kmap, full(s), 0, kb * 128, h, b);
            tma_load_4d(st + OFF_V + g * V_BYTES, &vmap, full(s), kb * 128, 0, h, b);
            tma_load_4d(st + OFF_V + g * V_BYTES + V_BYTES / 2, &vmap, full(s), kb * 128 + 64, 0, h, b);
            tma_load_3d(st + OFF_MB + g * MB_BYTES, &mmap, full(s), kb * 128, b, 0);
          }
          if (p.has_bias) {  // the transposed bias [h][k][q]: 128 keys x (two boxes of 64 queries)
            tma_load_3d(st + OFF_BIAS, &bmap, full(s), qb * 128, kb * 128, h);
            tma_load_3d(st + OFF_BIAS + BIAS_BYTES / 2, &bmap, full(s), qb * 128 + 64, kb * 128, h);
          }
        }
      }
      // loads still in flight (all consumed unless a role gave up)
      for (int j = std::max(0, it - STAGES); j < it; ++j) mbar_wait_drain(full(j % STAGES), (j / STAGES) & 1, p.err);
      if (uit > 0) mbar_wait_drain(q_full, (uit - 1) & 1, p.err);
    }
  } else if (warp == 1) {
    // ---- MMA issue (warp-uniform loop, one elected lane per instruction) ----
    const uint32_t idesc_qk = idesc_f16_f32(128, 128), idesc_pv = idesc_f16_f32(128, 32);
    const uint32_t idesc_bias = idesc_f16_f32(128, 128);  // B = the bias tile, keys x queries, K-major
    int it = 0, uit = 0;
    bool ok = true;
    auto qk = [&](int g, int tile) -> bool {
      // S_g = I . bias (the tile's bias rows, exactly: K runs over the 128 queries, one-hot A from
      // TMEM) + Q_g K_g^T over the 32 head channels (two K = 16 steps in the 64-byte rows)
      if (!warp_wait(s_free(g), (tile & 1) ^ 1, abort_flag, p.err, kErrWaitMma)) return false;
      tc_fence_after();
      const uint32_t st = sbase + (tile % STAGES) * STAGE_BYTES;
      const uint64_t qd = sdesc_k_sw64(sbase + OFF_Q + g * Q_BYTES), kd = sdesc_k_sw64(st + OFF_K + g * K_BYTES);
      const uint32_t d = tmem + g * TM_GROUP;
      if (p.has_bias) {
        // the tile holds bias[q][k] as rows k of 128 queries (two 64-query boxes, 128B-swizzled)
        const uint64_t bd = sdesc_k_sw128(st + OFF_BIAS);
        umma_ts_first(d, tmem + tm_identity(0), bd, idesc_bias);
#pragma unroll
        for (int ks = 1; ks < 8; ++ks)
          umma_ts_acc(d, tmem + tm_identity(ks), desc_add(bd, (ks >> 2) * (BIAS_BYTES / 2)) + (ks & 3) * 2,
                      idesc_bias);
        umma_acc(d, qd, kd, idesc_qk);
      } else {
        umma_first(d, qd, kd, idesc_qk);
      }
      umma_acc(d, qd + 2, kd + 2, idesc_qk);
      umma_commit(s_full(g));
      return true;
    };
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x, ++uit) {
      if (!warp_wait(q_full, uit & 1, abort_flag, p.err, kErrWaitMma)) break;
      // the first key block's scores
      if (!warp_wait(full(it % STAGES), (it / STAGES) & 1, abort_flag, p.err, kErrWaitMma)) break;
      tc_fence_after();
      if (!qk(0, it) || !qk(1, it)) break;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        if (kb + 1 < nkb) {
          // the next key block's scores run while this block's softmax works
          const int nx = it + 1;
          if (!warp_wait(full(nx % STAGES), (nx / STAGES) & 1, abort_flag, p.err, kErrWaitMma) || !qk(0, nx) ||
              !qk(1, nx)) {
            ok = false;
            break;
          }
        } else {
          umma_commit(q_empty);  // every score product of this unit has been issued
        }
        const uint32_t st = sbase + s * STAGE_BYTES;
        for (int g = 0; g < 2; ++g) {
          if (!warp_wait(p_full(g), it & 1, abort_flag, p.err, kErrWaitMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + g * TM_GROUP + TM_O, a = tmem + g * TM_GROUP + TM_P;
          const uint64_t v0 = sdesc_k_sw128(st + OFF_V + g * V_BYTES);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint64_t vd = desc_add(v0, (ks >> 2) * (V_BYTES / 2)) + (ks & 3) * 2;
            if (kb == 0 && ks == 0)
              umma_ts_first(d, a, vd, idesc_pv);
            else
              umma_ts_acc(d, a + 8 * ks, vd, idesc_pv);
          }
          umma_commit(o_done(g));
        }
        if (!ok) break;
        umma_commit(empty(s));
      }
    }
    umma_commit(drain);
    mbar_wait_drain(drain, 0, p.err);
  } else {
    // ---- softmax: group g owns batch row 2 bp + g; thread = one query row (TMEM lane) ----
    const int g = (warp - 2) >> 2, qd = warp & 3, r = qd * 32 + lane;
    const uint32_t lane_off = static_cast<uint32_t>(qd * 32) << 16;
    const uint32_t t_s = tmem + lane_off + g * TM_GROUP, t_p = t_s + TM_P, t_o = t_s + TM_O;
    const int C = p.channels;
    int it = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok && u < p.units; u += gridDim.x) {
      const int qb = u % p.nqb, rest = u / p.nqb, bp = rest % p.nbp, h = rest / p.nbp;
      const int64_t b = 2 * bp + g, qrow = static_cast<int64_t>(qb) * 128 + r;
      const int *flags = p.flags + (b < p.batch ? b : 0) * static_cast<int64_t>(nkb);
      float m_run = -INFINITY, l_run = 0.f;
      uint32_t flag_bits = 0;
      for (int kb = 0; kb < nkb; ++kb, ++it) {
        const int s = it % STAGES;
        // masked keys or keys past Q in this block (a row past the batch reads row 0's flags: its
        // scores are zeros and never stored); 32 blocks' flags at a time, one per lane
        if ((kb & 31) == 0) flag_bits = __ballot_sync(kFull, kb + lane < nkb && __ldg(flags + kb + lane) != 0);
        const bool flagged = (flag_bits >> (kb & 31)) & 1u;
        if (!warp_wait(s_full(g), it & 1, abort_flag, p.err, kErrWaitEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t t[128];
        {
          uint32_t (&c0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&t[0]);
          uint32_t (&c1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&t[32]);
          uint32_t (&c2)[32] = *reinterpret_cast<uint32_t(*)[32]>(&t[64]);
          uint32_t (&c3)[32] = *reinterpret_cast<uint32_t(*)[32]>(&t[96]);
          tmem_ld32(t_s, c0);
          tmem_ld32(t_s + 32, c1);
          tmem_ld32(t_s + 64, c2);
          tmem_ld32(t_s + 96, c3);
          tmem_ld_wait();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(s_free(g));  // S may be overwritten by the next block's scores
        // S = q.k / sqrt(d) + bias, in base 2.  The reference adds 1e9 (mask - 1) and clamps to
        // +-1e8 (here in base-2 units): exactly that where the block has masked keys (keys past Q
        // drop out); elsewhere a logit can only reach the clamp if the row maximum is within
        // 256 of it, and only then is every logit clamped.
        float mx = -INFINITY;
        if (flagged) {
          if (!warp_wait(full(s), (it / STAGES) & 1, abort_flag, p.err, kErrWaitEpilogue)) {
            ok = false;
            break;
          }
          const float *mb = reinterpret_cast<const float *>(smem + s * STAGE_BYTES + OFF_MB + g * MB_BYTES);
          const int64_t keys_left = p.queries - static_cast<int64_t>(kb) * 128;
          const int kvalid = keys_left < 128 ? static_cast<int>(keys_left) : 128;
#pragma unroll
          for (int c4 = 0; c4 < 32; ++c4) {
            const float4 m4 = *reinterpret_cast<const float4 *>(mb + 4 * c4);
            const float mk[4] = {m4.x, m4.y, m4.z, m4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int key = 4 * c4 + e;
              float v = fminf(fmaxf(__uint_as_float(t[key]) + mk[e], -kClamp), kClamp);
              if (key >= kvalid) v = -INFINITY;
              t[key] = __float_as_uint(v);
              mx = fmaxf(mx, v);
            }
          }
        } else {
          float m8[8];  // eight independent chains, not one 128 long
#pragma unroll
          for (int i = 0; i < 8; ++i) m8[i] = __uint_as_float(t[i]);
#pragma unroll
          for (int key = 8; key < 128; ++key) m8[key & 7] = fmaxf(m8[key & 7], __uint_as_float(t[key]));
          mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])), fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
          if (__any_sync(kFull, mx > kClamp || mx < 256.f - kClamp)) {
            mx = -INFINITY;
#pragma unroll
            for (int key = 0; key < 128; ++key) {
              const float v = fminf(fmaxf(__uint_as_float(t[key]), -kClamp), kClamp);
              t[key] = __float_as_uint(v);
              mx = fmaxf(mx, v);
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(s));  // this warp is done with the stage's mask
        // lazy maximum: move it (and rescale O and the sum) only when it grows by more than 2^8
        const bool move = mx > m_run + kLazyRescale;
        const float m_new = move ? mx : m_run;
        const float alpha = move ? ex2f(m_run - m_new) : 1.f;  // 0 on the first block (m_run = -inf)
        // the exponentials, into registers, while the previous block's P . V may still run
        float2 sum4[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
        const float2 neg_m = make_float2(-m_new, -m_new);
#pragma unroll
        for (int i = 0; i < 64; ++i) {
          const float2 x = f2add(make_float2(__uint_as_float(t[2 * i]), __uint_as_float(t[2 * i + 1])), neg_m);
          const float2 pe = make_float2(ex2f(x.x), ex2f(x.y));
          sum4[i & 3] = f2add(sum4[i & 3], pe);
          t[i] = pack_half2(pe.x, pe.y);  // P pairs overwrite the consumed logits
        }
        const float2 sum2 = f2add(f2add(sum4[0], sum4[1]), f2add(sum4[2], sum4[3]));
        if (kb > 0) {
          // P of the previous block has been consumed and O holds its sum
          if (!warp_wait(o_done(g), (it - 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (__any_sync(kFull, move)) {
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
              uint32_t o[16];
              tmem_ld16(t_o + 16 * hf, o);
              tmem_ld_wait();
#pragma unroll
              for (int i = 0; i < 16; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
              tmem_st16(t_o + 16 * hf, o);
            }
            tmem_st_wait();
          }
        }
#pragma unroll
        for (int c = 0; c < 4; ++c) tmem_st16(t_p + 16 * c, &t[16 * c]);
        tmem_st_wait();
        l_run = l_run * alpha + (sum2.x + sum2.y);
        m_run = m_new;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(p_full(g));
      }
      if (!ok) break;
      // ---- the unit's output rows: O / l times the gate -> weighted[b * Q + q][32 h ..] ----
      if (!warp_wait(o_done(g), (it - 1) & 1, abort_flag, p.err, kErrWaitEpilogue)) break;
      tc_fence_after();
      uint32_t o[32];
      tmem_ld32(t_o, o);
      tmem_ld_wait();
      tc_fence_before();
      if (b < p.batch && qrow < p.queries) {
        const int64_t row = b * p.queries + qrow;
        const float inv = 1.f / l_run;
        const uint4 *g4 = reinterpret_cast<const uint4 *>(p.gate + row * C + 32 * h);
        uint4 *w4 = reinterpret_cast<uint4 *>(p.weighted + row * C + 32 * h);
#pragma unroll
        for (int w = 0; w < 4; ++w) {
          float gv[8];
          unpack8<__half>(__ldg(g4 + w), gv);
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            pk[i] = pack_half2(__uint_as_float(o[8 * w + 2 * i]) * inv * gv[2 * i],
                               __uint_as_float(o[8 * w + 2 * i + 1]) * inv * gv[2 * i + 1]);
          w4[w] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
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

}  // namespace attn

using namespace attn;

// Column blocks of the projection GEMM: [q | k | v | g] (C each) then the pair bias, padded
// to 64 columns; the column tile is the widest multiple of 32 (<= 256) dividing the total.
static int64_t attention_proj_cols(int64_t c) { return 4 * c + 64; }
static int attention_proj_bn(int64_t cols) {
  for (int bn : {256, 192, 160, 128, 96, 64})
    if (cols % bn == 0) return bn;
  return 64;
}

AttentionLayout attention_layout(int64_t batch, int64_t queries, int64_t channels, int64_t heads, bool bias) {
  AttentionLayout L;
  L.b = batch;
  L.q = queries;
  L.c = channels;
  L.h = heads;
  L.bias = bias;
  L.rows = batch * queries;
  L.pitch = align_up(queries, 64);
  L.k_pad = align_up(channels, 64);
  L.cols = attention_proj_cols(channels);
  L.bn = attention_proj_bn(L.cols);
  L.o_cols = linear_cols_pad(channels);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes, 256);
    return at;
  };
  L.off_w = take((size_t)L.k_pad * L.cols * 2);
  L.off_scale = take((size_t)L.cols * 4);
  L.off_bvec = take((size_t)L.cols * 4);
  L.off_wo = take((size_t)L.k_pad * L.o_cols * 2);
  L.off_wo_scale = take((size_t)L.o_cols * 4);
  L.off_wo_bias = take((size_t)L.o_cols * 4);
  L.off_ln = take((size_t)channels * 2 * 4);
  L.off_xn = take((size_t)L.rows * channels * 2);  // the normalised rows, later the weighted values
  L.off_q = take((size_t)L.rows * channels * 2);
  L.off_k = take((size_t)L.rows * channels * 2);
  L.off_vt = take((size_t)batch * heads * 32 * L.pitch * 2);
  L.off_g = take((size_t)L.rows * channels * 2);
  L.off_pb = take(bias ? (size_t)heads * queries * L.pitch * 2 : 0);
  L.off_mb = take((size_t)batch * L.pitch * 4);
  L.off_flags = take((size_t)batch * ((queries + 127) / 128) * 4);
  L.total = off;
  return L;
}

af2_status attention_launch(af2_ctx *ctx, const AttentionLayout &L, int transpose, const void *x, int x_dtype,
                            const float *mask, const float *packed, double eps, int residual, void *out,
                            int out_dtype, void *workspace, cudaStream_t stream) {
  uint8_t *ws = static_cast<uint8_t *>(workspace);
  const int64_t C = L.c, H = L.h, B = L.b, Q = L.q;
  // packAttentionWeights order (attention.ts:179-201): queryNorm scale / offset, query, key, value,
  // gating weights [C, C] ([in, out]), gating bias, output weight [C, C], output bias, pair projection [C, H].
  const float *ln_s = packed, *ln_o = ln_s + C, *wq = ln_o + C, *wk = wq + C * C, *wv = wk + C * C,
              *wg = wv + C * C, *bg = wg + C * C, *wo = bg + C, *bo = wo + C * C, *wb = bo + C;
  af2_status st;
  // the prepared weights: the layout's prefix [0, off_xn), in the weight cache or the workspace
  WeightKey key;
  key.kind = kWeightsAttention;
  key.ptr[0] = packed;
  key.dim[0] = C;
  key.dim[1] = H;
  key.dim[2] = L.bias ? 1 : 0;
  PreparedRegion pw;
  if ((st = prepared_region(ctx, key, L.off_xn, ws, true, &pw)) != AF2_OK) return st;
  uint8_t *wp = pw.base;
  float *scale = reinterpret_cast<float *>(wp + L.off_scale), *bvec = reinterpret_cast<float *>(wp + L.off_bvec);
  float *wo_scale = reinterpret_cast<float *>(wp + L.off_wo_scale), *wo_bias = reinterpret_cast<float *>(wp + L.off_wo_bias);
  float *ln = reinterpret_cast<float *>(wp + L.off_ln);
  if (pw.fresh) {
    const float qscale = kLog2e / std::sqrt(32.f);
    auto f32m = [](const float *p) { return af2_matrix{AF2_WEIGHTS_F32, 0, p, nullptr}; };
    PrepJob jobs[6] = {
        {f32m(wq), C, C, L.k_pad, C, qscale, wp + L.off_w, scale, 0, L.cols},
        {f32m(wk), C, C, L.k_pad, C, 1.f, wp + L.off_w, scale, C, L.cols},
        {f32m(wv), C, C, L.k_pad, C, 1.f, wp + L.off_w, scale, 2 * C, L.cols},
        {f32m(wg), C, C, L.k_pad, C, 1.f, wp + L.off_w, scale, 3 * C, L.cols},
        {f32m(wo), C, C, L.k_pad, L.o_cols, 1.f, wp + L.off_wo, wo_scale, 0, 0},
        // the pair-bias columns (zeros without a bias): the padded tail of the projection
        {f32m(L.bias ? wb : wq), C, L.bias ? H : 0, L.k_pad, L.cols - 4 * C, kLog2e, wp + L.off_w, scale, 4 * C,
         L.cols},
    };
    if ((st = prepare_matrices(ctx, jobs, 6, stream)) != AF2_OK) return st;
    VectorSegments vs{};
    vs.add(nullptr, 0, 3 * C, bvec);
    vs.add(bg, C, C, bvec + 3 * C);
    vs.add(nullptr, 0, L.cols - 4 * C, bvec + 4 * C);
    vs.add(bo, C, L.o_cols, wo_bias);
    vs.add(ln_s, C, C, ln);
    vs.add(ln_o, C, C, ln + C);
    if ((st = pad_vectors(ctx, vs, stream)) != AF2_OK) return st;
  }
  __half *xn = reinterpret_cast<__half *>(ws + L.off_xn);
  if (C == 128 && reinterpret_cast<uintptr_t>(x) % 16 == 0) {
    const int warps = 8;
    const unsigned blocks = (unsigned)((L.rows + 4 * warps - 1) / (4 * warps));
    LaunchScope scope(ctx, stream, kProfAttentionNormalize);
    if (x_dtype == AF2_F32)
      attn_norm128_kernel<float><<<blocks, warps * 32, 0, stream>>>(static_cast<const float *>(x), L.rows, B, Q,
                                                                    transpose, ln, ln + C, (float)eps, xn);
    else if (x_dtype == AF2_BF16)
      attn_norm128_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, stream>>>(
          static_cast<const __nv_bfloat16 *>(x), L.rows, B, Q, transpose, ln, ln + C, (float)eps, xn);
    else
      attn_norm128_kernel<__half><<<blocks, warps * 32, 0, stream>>>(static_cast<const __half *>(x), L.rows, B, Q,
                                                                     transpose, ln, ln + C, (float)eps, xn);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention LayerNorm");
  } else {
    const int warps = 8;
    const unsigned blocks = (unsigned)((L.rows + warps - 1) / warps);
    LaunchScope scope(ctx, stream, kProfAttentionNormalize);
    if (x_dtype == AF2_F32)
      attn_norm_kernel<float><<<blocks, warps * 32, 0, stream>>>(static_cast<const float *>(x), L.rows, (int)C, B, Q,
                                                                 transpose, ln, ln + C, (float)eps, xn);
    else if (x_dtype == AF2_BF16)
      attn_norm_kernel<__nv_bfloat16><<<blocks, warps * 32, 0, stream>>>(
          static_cast<const __nv_bfloat16 *>(x), L.rows, (int)C, B, Q, transpose, ln, ln + C, (float)eps, xn);
    else
      attn_norm_kernel<__half><<<blocks, warps * 32, 0, stream>>>(static_cast<const __half *>(x), L.rows, (int)C, B,
                                                                  Q, transpose, ln, ln + C, (float)eps, xn);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention LayerNorm");
  }
  float *mb = reinterpret_cast<float *>(ws + L.off_mb);
  {
    LaunchScope scope(ctx, stream, kProfAttentionNormalize);
    attn_mask_kernel<<<(unsigned)((B * Q + 255) / 256), 256, 0, stream>>>(mask, B, Q, transpose, L.pitch, mb);
    const int nkb = (int)((Q + 127) / 128);
    attn_flag_kernel<<<(unsigned)((B * nkb + 7) / 8), 256, 0, stream>>>(mask, B, Q, transpose, nkb,
                                                                       reinterpret_cast<int *>(ws + L.off_flags));
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention mask");
  }
  AttentionProjection ap;
  ap.q = ws + L.off_q;
  ap.k = ws + L.off_k;
  ap.vt = ws + L.off_vt;
  ap.g = ws + L.off_g;
  ap.bias = L.bias ? ws + L.off_pb : nullptr;
  ap.queries = Q;
  ap.pitch = L.pitch;
  ap.channels = C;
  ap.heads = H;
  {
    LinearOperands op;
    op.a = xn;
    op.lda = C;
    op.inner = C;
    op.w = wp + L.off_w;
    op.scale = scale;
    op.bias = bvec;
    op.rows = L.rows;
    op.cols = L.cols;
    op.bn = L.bn;
    op.attention = &ap;
    op.prof = kProfAttentionProject;
    if ((st = linear_launch(ctx, op, stream)) != AF2_OK) return st;
  }
  // ---- flash loop ----
  {
    CUtensorMap qmap, kmap, vmap, bmap, mmap;
    std::memset(&bmap, 0, sizeof bmap);
    const uint64_t qk_dims[4] = {32, (uint64_t)Q, (uint64_t)H, (uint64_t)B};
    const uint64_t qk_strides[3] = {64, (uint64_t)Q * 64, (uint64_t)H * Q * 64};
    const uint32_t qk_box[4] = {32, 128, 1, 1};
    const uint64_t v_dims[4] = {(uint64_t)Q, 32, (uint64_t)H, (uint64_t)B};
    const uint64_t v_strides[3] = {(uint64_t)L.pitch * 2, (uint64_t)32 * L.pitch * 2, (uint64_t)H * 32 * L.pitch * 2};
    const uint32_t v_box[4] = {64, 32, 1, 1};
    if (!encode_map_4d(&qmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_q, qk_dims, qk_strides, qk_box,
                       CU_TENSOR_MAP_SWIZZLE_64B) ||
        !encode_map_4d(&kmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_k, qk_dims, qk_strides, qk_box,
                       CU_TENSOR_MAP_SWIZZLE_64B) ||
        !encode_map_4d(&vmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_vt, v_dims, v_strides, v_box,
                       CU_TENSOR_MAP_SWIZZLE_128B) ||
        !encode_map_3d(&mmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, mb, Q, B, 1, L.pitch * 4, (uint64_t)B * L.pitch * 4,
                       128, 1, 1, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        (L.bias && !encode_map_3d(&bmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, ws + L.off_pb, Q, Q, H, L.pitch * 2,
                                  (uint64_t)Q * L.pitch * 2, 64, 128, 1, CU_TENSOR_MAP_SWIZZLE_128B)))
      return fail(ctx, AF2_ERR_CUDA, "cuTensorMapEncodeTiled failed for the attention operands");
    FlashArgs a{};
    a.weighted = xn;  // the normalised rows are dead after the projection
    a.gate = reinterpret_cast<const __half *>(ws + L.off_g);
    a.flags = reinterpret_cast<const int *>(ws + L.off_flags);
    a.batch = B;
    a.queries = Q;
    a.channels = (int)C;
    a.heads = (int)H;
    a.nqb = (int)((Q + 127) / 128);
    a.nkb = a.nqb;
    a.nbp = (int)((B + 1) / 2);
    a.units = (int)(H * a.nbp * a.nqb);
    a.has_bias = L.bias ? 1 : 0;
    a.err = ctx->err_word;
    cudaError_t e = cudaFuncSetAttribute(attn_flash_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel attributes");
    const int grid = std::max(1, std::min(a.units, ctx->sm_count));
    LaunchScope scope(ctx, stream, kProfAttentionFlash);
    attn_flash_kernel<<<grid, THREADS, SMEM_BYTES, stream>>>(qmap, kmap, vmap, bmap, mmap, a);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(ctx, e, "attention kernel launch");
  }
  // ---- output projection, written (or added) to the source rows ----
  LinearOperands op;
  op.a = xn;
  op.lda = C;
  op.inner = C;
  op.w = wp + L.off_wo;
  op.scale = wo_scale;
  op.bias = wo_bias;
  op.rows = L.rows;
  op.cols = C;
  op.out = out;
  op.ldo = C;
  op.out_dtype = out_dtype;
  op.residual = residual;
  if (transpose) {
    op.transpose_q = Q;
    op.transpose_b = B;
  }
  op.prof = kProfAttentionOutput;
  return linear_launch(ctx, op, stream);
}

}  // namespace af2
