// block.cu -- the Evoformer pair block: encodeEvoformerPairBlock
// (src/evoformer/block.ts:1753-1805) as one C-ABI call on device tensors.
//
// The reference encodes, on one command encoder and with the pair as every
// op's residual target: the outer-product mean of the MSA (optional),
// triangle multiplication outgoing then incoming, triangle attention around
// the starting node then the ending node (the transposed view), and the pair
// transition.  Here the same six ops run back to back on one stream through
// their launchers, every update added into the pair in place, with the
// context's scratch grown once to the largest op's need.
#include <algorithm>
#include <string>

#include "af2_internal.h"

using namespace af2;

extern "C" af2_status af2_evoformer_pair_block(af2_ctx *ctx, const af2_pair_block_shape *shape,
                                               const af2_pair_block_weights *weights, const void *msa, int msa_dtype,
                                               const float *msa_mask, void *pair, int pair_dtype,
                                               const float *pair_mask, const af2_pair_block_options *options,
                                               void *stream) {
  if (!ctx) return AF2_ERR_INVALID_ARGUMENT;
  if (!shape || !weights) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "shape or weights is NULL");
  const bool with_opm = options ? options->include_outer_product_mean != 0 : true;
  const double eps = (options && options->epsilon != 0) ? options->epsilon : 1e-5;
  const int64_t n = shape->length, cz = shape->c_z;
  if (!pair || !pair_mask) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "pair or pair mask is NULL");
  if (with_opm && (!msa || !msa_mask || !weights->outer_product_mean))
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "the outer product mean needs the MSA, its mask and its weights");
  if (!weights->triangle_outgoing || !weights->triangle_incoming || !weights->attention_starting ||
      !weights->attention_ending)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a weight array is NULL");
  // every op's own validation, on the shapes the block gives it
  char message[256];
  af2_status st;
  const af2_triangle_shape ts{n, cz, shape->c_hidden};
  const int64_t tri_count = af2_triangle_weight_count(cz, shape->c_hidden);
  if ((st = af2_triangle_check(0, &ts, tri_count, eps, message, sizeof message)) != AF2_OK)
    return fail(ctx, st, std::string("triangle multiplication: ") + message);
  const af2_attention_shape as{n, n, cz, shape->pair_heads};
  const int64_t att_count = af2_attention_weight_count(&as, AF2_PAIR_BIAS_NORMALIZED_INPUT);
  if ((st = af2_attention_check(&as, AF2_PAIR_BIAS_NORMALIZED_INPUT, att_count, eps, message, sizeof message)) !=
      AF2_OK)
    return fail(ctx, st, std::string("triangle attention: ") + message);
  const af2_transition_shape trs{n * n, cz, shape->transition_hidden};
  if ((st = af2_transition_check(&trs, af2_transition_weight_count(cz, shape->transition_hidden), eps, message,
                                 sizeof message)) != AF2_OK)
    return fail(ctx, st, std::string("pair transition: ") + message);
  const af2_opm_shape os{shape->sequences, n, shape->c_m, shape->c_outer, cz};
  if (with_opm && (st = af2_opm_check(&os, af2_opm_weight_count(&os), message, sizeof message)) != AF2_OK)
    return fail(ctx, st, std::string("outer product mean: ") + message);
  const bool dtypes_ok = (pair_dtype == AF2_F32 || pair_dtype == AF2_F16 || pair_dtype == AF2_BF16) &&
                         (!with_opm || msa_dtype == AF2_F32 || msa_dtype == AF2_F16 || msa_dtype == AF2_BF16);
  if (!dtypes_ok) return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "dtype must be AF2_F32, AF2_F16 or AF2_BF16");
  const af2_transition_weights &tw = weights->pair_transition;
  if (!tw.layer_norm_scale || !tw.layer_norm_offset || !tw.first_bias || !tw.second_bias || !tw.first_weight.values ||
      !tw.second_weight.values)
    return fail(ctx, AF2_ERR_INVALID_ARGUMENT, "a pair transition weight is NULL");
  cudaSetDevice(ctx->device);
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;

  const OpmLayout lo = opm_layout(shape->sequences, n, shape->c_m, shape->c_outer, cz, 0, 0, 0,
                                  ctx->gemm_precision == AF2_GEMM_F32);
  const TriangleLayout lt = triangle_layout(n, cz, shape->c_hidden, 0, pair_dtype);
  const AttentionLayout la = attention_layout(n, n, cz, shape->pair_heads, true);
  const TransitionLayout lr = transition_layout(n * n, cz, shape->transition_hidden, pair_dtype);
  const size_t need = std::max({with_opm ? lo.total : size_t(0), lt.total, la.total, lr.total});
  if ((st = ensure(ctx, ctx->workspace, need, "pair block scratch")) != AF2_OK) return st;
  void *ws = ctx->workspace.ptr;

  if (with_opm &&
      (st = opm_launch(ctx, lo, msa, msa_dtype, msa_mask, weights->outer_product_mean, eps, 1e-3, 1, pair, pair_dtype,
                       ws, s)) != AF2_OK)
    return st;
  if ((st = triangle_launch(ctx, AF2_OUTGOING, lt, pair, pair_dtype, pair_mask, weights->triangle_outgoing, eps, 1,
                            pair, pair_dtype, ws, s)) != AF2_OK ||
      (st = triangle_launch(ctx, AF2_INCOMING, lt, pair, pair_dtype, pair_mask, weights->triangle_incoming, eps, 1,
                            pair, pair_dtype, ws, s)) != AF2_OK ||
      (st = attention_launch(ctx, la, 0, pair, pair_dtype, pair_mask, weights->attention_starting, eps, 1, pair,
                             pair_dtype, ws, s)) != AF2_OK ||
      (st = attention_launch(ctx, la, 1, pair, pair_dtype, pair_mask, weights->attention_ending, eps, 1, pair,
                             pair_dtype, ws, s)) != AF2_OK)
    return st;
  return transition_launch(ctx, lr, pair, pair_dtype, tw, eps, 1, pair, pair_dtype, ws, s);
}
