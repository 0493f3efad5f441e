// af2_internal.h -- host-side pieces shared by the C-ABI layer (api.cu) and
// the per-operator launchers (triangle.cu, ...).  Nothing here crosses the ABI.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

#include "../../include/af2cuda.h"

namespace af2 {

// Device-side scratch owned by a context: grown on demand, never shrunk.
struct DeviceBuffer {
  void *ptr = nullptr;
  size_t bytes = 0;
};

}  // namespace af2

namespace af2 {
// What a prepared-weights cache entry was made from: the op, its weight pointers and the
// dimensions and options the preparation depends on.
struct WeightKey {
  int kind = 0;
  const void *ptr[32] = {};
  int64_t dim[8] = {};
  bool operator==(const WeightKey &o) const;
};
struct CachedWeights {
  WeightKey key;
  DeviceBuffer buf;
};
enum WeightKind {
  kWeightsTriangle = 1, kWeightsOpm, kWeightsTransition, kWeightsAttention, kWeightsLinear, kWeightsTriangleTensors,
  kWeightsOpmTensors
};
}  // namespace af2

namespace af2 {
// Kernels the per-launch profiler distinguishes (labels follow the reference's
// dispatch labels, src/runtime/kernel-cost.ts:158-162).
enum ProfileKernel {
  kProfTrianglePrepare = 0,
  kProfTriangleRelayout,
  kProfTriangleProject,
  kProfTriangleContract,
  kProfTriangleOutput,
  kProfTransitionPrepare,
  kProfTransitionNormalize,
  kProfTransition,
  kProfDequant,
  kProfPrepare,
  kProfConvert,
  kProfLinear,
  kProfOpmNormalize,
  kProfOpmProject,
  kProfOpmCount,
  kProfOpmOuter,
  kProfOpmOutput,
  kProfOpmFused,
  kProfTransitionLinear,
  kProfAttentionNormalize,
  kProfAttentionProject,
  kProfAttentionFlash,
  kProfAttentionOutput,
  kProfCount
};
const char *profile_name(int id);
struct ProfilePending {
  int id;
  cudaEvent_t start, stop;
};
}  // namespace af2

struct af2_ctx {
  int device = 0;
  int sm_count = 0;
  int contract_pairs = 0;  // CTA pairs of the triangle contraction resident together (0: not queried)
  cudaStream_t stream = nullptr;
  unsigned int *err_word = nullptr;  // device word the kernels flag failures in
  af2::DeviceBuffer workspace;       // device-form scratch
  af2::DeviceBuffer staging[4];      // host-form device copies (z, mask, weights, out)
  cudaEvent_t ev_start = nullptr, ev_stop = nullptr;
  uint64_t launches = 0;
  bool profiling = false;
  std::vector<cudaEvent_t> free_events;
  std::vector<af2::ProfilePending> pending;
  uint64_t prof_launches[af2::kProfCount] = {};
  double prof_ms[af2::kProfCount] = {};
  uint64_t allocated = 0, peak = 0;
  std::string last_error;
  // Row-sharded operators (comm.cu): this rank's NCCL communicator and the
  // scratch of the distributed pair transpose.
  void *nccl_comm = nullptr;
  int nranks = 1, rank = 0;
  af2::DeviceBuffer shard_scratch;
  // The peers' shard scratch, mapped into this process (CUDA IPC) while `peer_of` is the
  // scratch allocation they were opened for; exchanges copy straight into it.
  void *peer_of = nullptr;
  std::vector<void *> peer_scratch;
  std::vector<cudaStream_t> copy_streams;  // one per peer: the exchange's copies run concurrently
  std::vector<cudaEvent_t> copy_events;
  int *sync_word = nullptr;                // device word the exchange barriers all-reduce
  bool ipc_failed = false;                 // mapping refused: exchanges use NCCL send/recv
  // failure detection: host waits on a stream that may hold collectives give up after this many
  // seconds (or at the communicator's first asynchronous error) and abort the communicator
  double comm_timeout_s = 600.0;
  bool comm_aborted = false;
  int gemm_precision = 0;                  // af2_gemm_precision: what the GEMMs that honour it multiply in
  // af2_set_weight_cache: prepared weights kept per weights pointer and shape, made once
  bool weight_cache = false;
  std::vector<af2::CachedWeights> cached_weights;
};

namespace af2 {

// Kernel-selection override from the environment (measurement of the alternatives a shape
// rule chooses between): the integer value of `name`, or `fallback` when unset or not a number.
int tuning_override(const char *name, int fallback);

// Sets ctx->last_error and returns `status`.
af2_status fail(af2_ctx *ctx, af2_status status, const std::string &message);
// Maps a CUDA error to AF2_ERR_CUDA (or AF2_ERR_OUT_OF_MEMORY) with context.
af2_status cuda_fail(af2_ctx *ctx, cudaError_t e, const char *what);
// Waits for `stream` on the host.  With a communicator: polls the stream and the communicator's
// asynchronous error with the context's deadline, and on an error or timeout aborts the
// communicator and returns AF2_ERR_NCCL (comm.cu).
af2_status comm_wait(af2_ctx *ctx, cudaStream_t stream, const char *what);
// Ensures `buf` holds at least `bytes` (256-byte aligned device memory).
af2_status ensure(af2_ctx *ctx, DeviceBuffer &buf, size_t bytes, const char *what);

// Where an op's prepared weights -- the prefix [0, bytes) of its scratch layout -- live.  With the
// context's weight cache on (and `allow` set), the cache entry for `key`: fresh when just made,
// so the caller prepares into it; else the workspace itself, always fresh.
struct PreparedRegion {
  uint8_t *base = nullptr;
  bool fresh = true;
};
af2_status prepared_region(af2_ctx *ctx, const WeightKey &key, size_t bytes, void *workspace, bool allow,
                           PreparedRegion *out);
void clear_weight_cache(af2_ctx *ctx);

// cuTensorMapEncodeTiled through the runtime's driver entry point.
bool encode_map_3d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, uint64_t d0, uint64_t d1,
                   uint64_t d2, uint64_t stride1_bytes, uint64_t stride2_bytes, uint32_t b0, uint32_t b1,
                   uint32_t b2, CUtensorMapSwizzle swizzle);
bool encode_map_4d(CUtensorMap *map, CUtensorMapDataType dtype, const void *base, const uint64_t (&dims)[4],
                   const uint64_t (&strides_bytes)[3], const uint32_t (&box)[4], CUtensorMapSwizzle swizzle);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Brackets one kernel launch with CUDA events on its stream while the
// context's profiler is on; counts the launch either way.
class LaunchScope {
 public:
  LaunchScope(af2_ctx *ctx, cudaStream_t stream, int id);
  ~LaunchScope();
  LaunchScope(const LaunchScope &) = delete;
  LaunchScope &operator=(const LaunchScope &) = delete;

 private:
  af2_ctx *ctx_;
  cudaStream_t stream_;
  int id_;
  cudaEvent_t start_ = nullptr;
};

// ---- triangle multiplication (triangle.cu) ----

struct TriangleLayout {
  int64_t n = 0, cz = 0, ch = 0;
  int64_t rows = 0;         // pair rows held here (n, or n / ranks when the pair is sharded by rows)
  int64_t block_rows = 0;   // output rows per block
  int64_t ranks = 1;        // channel shards of the contraction: the ranks of a row-sharded pair
  int64_t hq = 0;           // hidden channels per shard (128 / ranks)
  int64_t kp = 0;           // k pitch (elements) of the projected operands
  int64_t jp = 0;           // row pitch (elements) of the contracted block
  int64_t ab_rs = 0;        // row pitch (elements) of the projected operands [group][row][hq][kp]
  int64_t ab_rows = 0;      // rows of one channel group of the projected operands
  int64_t x_hs = 0;         // channel pitch (elements) of the contracted block
  bool pad_z = false;       // z is re-laid as f16 [P][128] before the kernels
  size_t off_w16 = 0, off_vec = 0, off_z16 = 0, off_a = 0, off_b = 0, off_x = 0;
  size_t off_a_all = 0, off_b_all = 0, off_x_all = 0;  // channel-sharded: exchanged operands and block
  size_t total = 0;
};

// One GPU: rows = 0.  A row-sharded pair: rows = n / ranks of them here; the
// layout then depends on the direction (the incoming product's k runs over
// the local rows).
TriangleLayout triangle_layout(int64_t n, int64_t cz, int64_t ch, int64_t block_rows, int z_dtype, int64_t rows = 0,
                               int direction = 0);

// Exchange of the channel-sharded contraction: block p of `send` (blocks
// `stride` bytes apart, `bytes` each) goes to rank p, and rank p's block for
// this rank lands in block p of `recv`; this rank's own block is left alone.
// One all-to-all of an exchange: block p of `send` goes to rank p, and rank p's block lands
// in block p of `recv` (blocks `stride` bytes apart, `bytes` each).  This rank's own block is
// not moved: the triangle kernels read and write it in place.
struct ShardTransfer {
  const void *send;
  void *recv;
  size_t stride, bytes;
};
// The exchange has two forms.  Direct: `direct` maps the peers' scratch (once per allocation)
// and reports whether copies can go straight into it; then `open` (every rank has finished
// reading its receive buffers), any number of `send`s issued between the kernels that produce
// their data, and `close` (every rank's data has landed).  Otherwise `exchange` moves whole
// transfers with NCCL send/recv.
struct TriangleShard {
  int ranks = 1, rank = 0;
  af2_status (*exchange)(af2_ctx *ctx, const ShardTransfer *transfers, int count, cudaStream_t stream) = nullptr;
  bool (*direct)(af2_ctx *ctx, cudaStream_t stream, af2_status *status) = nullptr;
  af2_status (*open)(af2_ctx *ctx, cudaStream_t stream) = nullptr;
  // `bytes` from `src` to the peer's scratch, at the offset `dst_local` has in this rank's
  af2_status (*send)(af2_ctx *ctx, const void *src, const void *dst_local, size_t bytes, int peer,
                     cudaStream_t stream) = nullptr;
  af2_status (*close)(af2_ctx *ctx, cudaStream_t stream) = nullptr;
  // the peer's shard scratch mapped into this process (valid after `direct` returned true), at
  // the same layout offsets as this rank's: kernels store their peer's pieces straight into it
  void *(*peer_base)(af2_ctx *ctx, int peer) = nullptr;
};

// Launches the whole op on `stream`; the workspace holds TriangleLayout::total bytes.
// cache_weights = false keeps the call from allocating a weight-cache entry (the static-scratch form).
// tensors (16 matrices in ORDER, f32 or q8 block; NULL: `packed` holds them) replaces `packed`.
af2_status triangle_launch(af2_ctx *ctx, int direction, const TriangleLayout &L, const void *z, int z_dtype,
                           const float *mask, const float *packed, double eps, int residual, void *out,
                           int out_dtype, void *workspace, cudaStream_t stream, const TriangleShard *shard = nullptr,
                           bool cache_weights = true, const af2_matrix *tensors = nullptr);

// ---- transition (transition.cu) ----

struct TransitionLayout {
  int64_t rows = 0, c = 0, h = 0;
  int64_t cp = 0;          // channels padded to 64 or 128 (the first GEMM's K, the second's N)
  int64_t hp = 0;          // hidden channels padded to 128 (the kernel works in 128-wide chunks)
  bool fast_in = false;    // 16-bit x with 16-byte rows: TMA straight into the kernel, LayerNorm in place
  int64_t chunk_rows = 0;  // rows per kernel launch (bounds the normalised copy otherwise)
  size_t off_w1 = 0, off_w2 = 0, off_vec = 0, off_xn = 0, total = 0;
  // Wide path (channels above 128 or hidden above 1024, e.g. the MSA transition at c_m = 256):
  // LayerNorm into an f16 copy, then the shared linear kernel twice, the hidden activations in
  // an HBM scratch per row chunk.
  bool wide = false;
  int64_t k1 = 0, n1 = 0, k2 = 0, n2 = 0;  // padded inner dimension / columns of the two GEMMs
  int64_t hid_pitch = 0;                   // hidden row pitch (elements)
  size_t off_s1 = 0, off_b1 = 0, off_s2 = 0, off_b2 = 0, off_hid = 0;
};

TransitionLayout transition_layout(int64_t rows, int64_t c, int64_t h, int x_dtype);

af2_status transition_launch(af2_ctx *ctx, const TransitionLayout &L, const void *x, int x_dtype,
                             const af2_transition_weights &w, double eps, int residual, void *out, int out_dtype,
                             void *workspace, cudaStream_t stream);

af2_status dequant_launch(af2_ctx *ctx, const af2_matrix &m, int64_t inner, int64_t cols, float *out,
                          cudaStream_t stream);

// ---- shared dense projection (gemm.cu) ----

// Destinations of the attention projection epilogue (attention.cu): q and k [b][h][j][32],
// v transposed [b][h][32][pitch], the gate [rows][channels], the pair bias transposed [h][k][pitch] (or NULL).
struct AttentionProjection {
  void *q = nullptr, *k = nullptr, *vt = nullptr, *g = nullptr, *bias = nullptr;  // f16
  int64_t queries = 0, pitch = 0, channels = 0, heads = 0;
};

// One tcgen05 GEMM D = A W over prepared weights, with its epilogue.
struct LinearOperands {
  const void *a = nullptr;        // f16 rows [rows][lda], the first `inner` columns used
  int64_t lda = 0;
  const void *w = nullptr;        // prepared weights [k_pad / 64][cols_pad][64] f16
  const float *scale = nullptr;   // per column (cols_pad entries)
  const float *bias = nullptr;    // per column (cols_pad entries)
  const float *row_scale = nullptr;  // per row, or NULL
  const float *row_mask = nullptr;   // OPM projection: per row
  int64_t rows = 0, inner = 0, cols = 0;
  void *out = nullptr;            // linear: [rows][ldo] of out_dtype
  int64_t ldo = 0;
  int out_dtype = AF2_F32;
  int relu = 0, residual = 0;
  bool opm_projection = false;    // columns [0, cols/2) -> left, the rest -> right (f16), times row_mask
  // opm_projection in the f32 precision mode: each value v is written as a split operand, left as
  // blocks (f16(v), f16(v), f16(v - f16(v))) and right as (f16(v), f16(v - f16(v)), f16(v)),
  // `split_stride_left` / `split_stride_right` elements apart, so that the outer-product GEMM
  // over the three blocks sums hi hi + hi lo + lo hi
  int64_t split_stride_left = 0, split_stride_right = 0;
  void *left = nullptr, *right = nullptr;
  // seq_pitch > 0: rows are m = i * kmajor_seqs + s, and left / right are written
  // sequence-contiguous: left [cols / 2][kmajor_rows][seq_pitch], right [rows][cols / 2][seq_pitch]
  int64_t kmajor_rows = 0, kmajor_seqs = 0, seq_pitch = 0;
  int prof = kProfLinear;
  int bn = 0;                     // column tile (a multiple of 32, at most 256); 0 = chosen from cols
  // the output row of row m = b * transpose_q + q is q * transpose_b + b (0: row m)
  int64_t transpose_q = 0, transpose_b = 0;
  const AttentionProjection *attention = nullptr;  // attention projection epilogue instead of `out`
};

// Tile width the GEMM uses for `cols` output columns, and the padded column count.
inline int64_t linear_tile_n(int64_t cols) { return cols >= 256 ? 256 : align_up(cols, 64); }
inline int64_t linear_cols_pad(int64_t cols) { return align_up(cols, linear_tile_n(cols)); }

// Prepares an [inner][cols] matrix as operand rows [inner_pad / 64][rows_total][64] starting at row
// row0 (rows_total 0 = cols_pad), and its per-column scales (times extra_scale) at scale_out[row0 ...].
af2_status prepare_matrix(af2_ctx *ctx, const af2_matrix &w, int64_t inner, int64_t cols, int64_t inner_pad,
                          int64_t cols_pad, float extra_scale, void *out, float *scale_out, cudaStream_t stream,
                          int64_t row0 = 0, int64_t rows_total = 0);
// Up to kMaxPrepJobs such preparations in one launch.
constexpr int kMaxPrepJobs = 6;
struct PrepJob {
  af2_matrix w;
  int64_t inner, cols, inner_pad, cols_pad;
  float extra_scale;
  void *out;
  float *scale_out;
  int64_t row0 = 0, rows_total = 0;
  const float *row_scale = nullptr;  // optional factor per inner row k (a LayerNorm gamma folded in)
  // 0: the f16 rounding of each scaled weight; 1: the f16 rounding of what that leaves (w - f16(w)),
  // the low half of a split operand (f32 precision mode)
  int part = 0;
};
af2_status prepare_matrices(af2_ctx *ctx, const PrepJob *jobs, int count, cudaStream_t stream);
// Up to 8 zero-padded vector copies done by one launch.
struct VectorSegments {
  const float *src[8];
  float *dst[8];
  int n[8], n_pad[8];
  int count;
  void add(const float *s, int64_t len, int64_t len_pad, float *d) {
    src[count] = s;
    dst[count] = d;
    n[count] = static_cast<int>(len);
    n_pad[count] = static_cast<int>(len_pad);
    ++count;
  }
};
af2_status pad_vectors(af2_ctx *ctx, const VectorSegments &v, cudaStream_t stream);
af2_status pad_vector(af2_ctx *ctx, const float *src, int64_t n, int64_t n_pad, float *dst, cudaStream_t stream);
af2_status convert_rows_f16(af2_ctx *ctx, const void *src, int dtype, int64_t rows, int64_t inner, int64_t inner_pad,
                            void *dst, cudaStream_t stream);
af2_status linear_launch(af2_ctx *ctx, const LinearOperands &op, cudaStream_t stream);

struct LinearLayout {
  int64_t k_pad = 0, cols_pad = 0;
  bool convert = false;  // A goes through an f16 copy first
  size_t off_w = 0, off_scale = 0, off_bias = 0, off_a = 0, total = 0;
};

LinearLayout linear_layout(int64_t rows, int64_t inner, int64_t cols, int a_dtype);
af2_status linear_run(af2_ctx *ctx, const LinearLayout &L, int64_t rows, int64_t inner, int64_t cols, const void *a,
                      int a_dtype, const af2_matrix &weight, const float *bias, int activation, int residual,
                      void *out, int out_dtype, void *workspace, cudaStream_t stream);

// ---- outer-product mean (opm.cu) ----

struct OpmLayout {
  int64_t s = 0, n = 0, cm = 0, c = 0, cz = 0;
  int64_t rows = 0, row0 = 0;  // output residues i held here (all n unless the pair is sharded)
  int64_t cmp = 0;          // c_m padded to 64
  int64_t block_rows = 0;   // residues i per output block (a multiple of 4)
  int out_shift = 0;        // outer is stored times 2^-out_shift (2^out_shift >= S)
  size_t off_wlr = 0, off_wlr_scale = 0, off_wlr_bias = 0, off_wo = 0, off_wo_scale = 0, off_wo_bias = 0;
  bool fused = false;        // outer product and output projection in one kernel (no outer scratch)
  bool split = false;        // f32 precision mode: every GEMM operand as an f16 hi / lo pair, K tripled
  int64_t seq_pitch = 0;    // fused: left [c][rows][seq_pitch] and right [n][c][seq_pitch], K-major
  size_t off_ln = 0, off_xn = 0, off_mask = 0, off_left = 0, off_right = 0, off_rowscale = 0, off_outer = 0;
  // per-tensor weights: the decoded small tensors (LayerNorm, W_left, W_right, biases) in f32,
  // read only by the preparation, which runs before the kernels that reuse this region
  size_t off_stage = 0;
  size_t total = 0;
};

// rows < n: this rank's residues [row0, row0 + rows) of a row-sharded pair.
OpmLayout opm_layout(int64_t s, int64_t n, int64_t cm, int64_t c, int64_t cz, int64_t row_block, int64_t rows = 0,
                     int64_t row0 = 0, bool split = false);

// Row-sharded OPM: this rank's block of the right operand is all-gathered in place.
struct OpmExchange {
  int rank = 0;
  bool m_local = false;  // m holds only this rank's residue columns [S][rows][c_m]
  af2_status (*all_gather)(af2_ctx *ctx, void *full, size_t bytes_per_rank, cudaStream_t stream) = nullptr;
};

af2_status opm_launch(af2_ctx *ctx, const OpmLayout &L, const void *m, int m_dtype, const float *mask,
                      const float *packed, double ln_eps, double norm_eps, int residual, void *out, int out_dtype,
                      void *workspace, cudaStream_t stream, const OpmExchange *exchange = nullptr,
                      const af2_matrix *tensors = nullptr);
// tensors (8 matrices in packOuterProductMeanWeights order, f32 or q8 block; NULL: `packed` holds
// them) replaces `packed`.

// ---- gated multi-head attention (attention.cu) ----

struct AttentionLayout {
  int64_t b = 0, q = 0, c = 0, h = 0;  // batch rows, queries (= keys), channels, heads (head dimension 32)
  bool bias = false;                   // pair bias from the normalised input (needs b == q)
  int64_t rows = 0;                    // b * q
  int64_t pitch = 0;                   // key pitch of the transposed values, the bias and the mask (64-aligned)
  int64_t k_pad = 0, cols = 0, o_cols = 0;
  int bn = 0;                          // column tile of the projection GEMM
  size_t off_w = 0, off_scale = 0, off_bvec = 0, off_wo = 0, off_wo_scale = 0, off_wo_bias = 0, off_ln = 0;
  size_t off_xn = 0, off_q = 0, off_k = 0, off_vt = 0, off_g = 0, off_pb = 0, off_mb = 0, off_flags = 0, total = 0;
};

AttentionLayout attention_layout(int64_t batch, int64_t queries, int64_t channels, int64_t heads, bool bias);

af2_status attention_launch(af2_ctx *ctx, const AttentionLayout &L, int transpose, const void *x, int x_dtype,
                            const float *mask, const float *packed, double eps, int residual, void *out,
                            int out_dtype, void *workspace, cudaStream_t stream);

// ---- row-sharded operators (comm.cu) ----

void comm_destroy(af2_ctx *ctx);

}  // namespace af2
