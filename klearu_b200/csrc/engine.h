// engine.h -- internal interfaces between the C-ABI layer (api.cu) and the
// kernel translation units of the klearu B200 engine.
#pragma once

#include <cstdint>

#include <cuda.h>

#include "common.cuh"

namespace kl {

// Process-wide count of kernels launched by this library (defined in api.cu).
void count_launch(unsigned n = 1);
// err |= bits, in stream order (a host-side failure reported like a kernel's).
void flag_error(int* err, int bits, cudaStream_t st);

// ---------------------------------------------------------------------------
// Hash families on the device.
// ---------------------------------------------------------------------------
struct TcPlanes;
struct DevHash {
  int kind = 0, d = 0, k = 0, L = 0, w = 0, bpw = 0, bin_size = 0;
  int LK = 0;           // L*K projections (SIMHASH / SRP)
  int dpad = 0;         // row pitch of `planes` (bytes, multiple of 16)
  int lkpad = 0;        // row pitch of `planesT` (bytes, multiple of 16)
  int8_t* planes = nullptr;     // [LK][dpad]  projection rows (SIMHASH, SRP as dense ternary)
  int8_t* planesT = nullptr;    // [d][lkpad]  transposed, for sparse inputs
  uint32_t* windows = nullptr;  // [L][K][w]   (WTA, DWTA)
  uint8_t* fallback = nullptr;  // [L][K]      DWTA sparse fallback position
  uint32_t* perms = nullptr;    // [L][d]      (MINHASH)
  // SIMHASH / SRP: non-zero entries of each projection in dimension order,
  // for the tiled dense kernel.  Dimensions are cut into tiles of PL_T; an
  // entry is (dim % PL_T) | 0x8000 when the coefficient is -1.  Projection tb owns plist[poff[tb*(nt+1)] ..
  // poff[tb*(nt+1)+nt]) and tile ti starts at poff[tb*(nt+1)+ti].
  uint16_t* plist = nullptr;
  uint32_t* poff = nullptr;     // [LK][nt+1]
  int nt = 0;                   // ceil(d / PL_T)
  const TcPlanes* tc = nullptr; // host-side: the tensor-core projection's planes (SIMHASH / SRP), or null
};

// Planes of the tensor-core SimHash / SRP projection (hash_tc.cu): exact bf16
// copies of the ternary planes, [H * Nh][dpad] with table group g in rows
// [g * Nh, g * Nh + tph * k), and their TMA descriptor.
struct TcPlanes {
  int H = 0, tph = 0, Nh = 0, kc = 0, dpad = 0, nst = 0;
  int mode = KL_PROJ_AUTO;
  bool ready = false;
  const void* planes = nullptr;  // device bf16 [H * Nh][dpad]
  int* err = nullptr;            // device error word
  alignas(64) CUtensorMap map;
};
bool tc_plane_layout(int d, int k, int L, TcPlanes* tp);
bool tc_plane_map(TcPlanes* tp);
constexpr int PL_T = 640;       // dimensions per staged tile (< 2^15)

// Dense input: element (i, j) of row i at X[i*ld_row + j*ld_elem], as f32 or bf16.
struct DenseIn {
  const void* X;
  int dtype;
  int64_t ld_row, ld_elem;
  int n;
};
// CSR input with sorted unique column indices.
struct SparseIn {
  const int32_t* rowptr;
  const uint32_t* idx;
  const float* val;
  int n;
};
// Hash outputs (each nullable): codes[i*L+t], min_abs[i*L+t] (SIMHASH/SRP),
// bkt[t*bkt_ld + i] = code & nb_mask (bucket index, 16 bits).
struct HashOut {
  uint64_t* codes = nullptr;
  float* min_abs = nullptr;
  uint16_t* bkt = nullptr;
  int64_t bkt_ld = 0;
  uint32_t nb_mask = 0;
};

void launch_hash_dense(const DevHash& h, const DenseIn& in, const HashOut& out, cudaStream_t st);
// The tensor-core SimHash / SRP projection of bf16 rows; false (nothing launched)
// when the input or the hash does not qualify.
bool launch_proj_tc(const DevHash& h, const DenseIn& in, const HashOut& out, int* err, cudaStream_t st);
void launch_hash_sparse(const DevHash& h, const SparseIn& in, const HashOut& out, cudaStream_t st);

// ---------------------------------------------------------------------------
// Bucket tables: L x nb buckets of `cap` ids each.
// ---------------------------------------------------------------------------
struct DevTables {
  int L = 0, nb = 0, cap = 0, type = 0;
  uint32_t* ids = nullptr;  // [L][nb][cap]
  uint32_t* len = nullptr;  // [L][nb]
  uint64_t* cnt = nullptr;  // [L][nb] total insertions (reservoir)
};

// Scratch for a batched insert of up to `n` items.
struct InsertScratch {
  uint32_t* chunk_cnt = nullptr;  // [L][nchunks][nb]
  uint32_t* total = nullptr;      // [L][nb]
  uint32_t* base = nullptr;       // [L][nb] first slot of the new items (FIFO)
  uint32_t* skip = nullptr;       // [L][nb] new items dropped at the front (FIFO)
  unsigned long long* temp = nullptr;  // [L][nb][cap] packed (rank, id) (reservoir)
};
constexpr int INSERT_CHUNK = 1024;
size_t insert_scratch_bytes(const DevTables& T, int n);
void carve_insert_scratch(const DevTables& T, int n, void* base, InsertScratch* s);

// n sequential inserts: item i has id ids[i] (ids == nullptr: id = i) and
// bucket bkt[t*bkt_ld + i] in table t.
void launch_tables_insert(const DevTables& T, const uint32_t* ids, const uint16_t* bkt,
                          int64_t bkt_ld, int n, const InsertScratch& s, int* err,
                          cudaStream_t st);
void launch_tables_clear(const DevTables& T, cudaStream_t st);
void launch_tables_remove(const DevTables& T, const uint32_t* ids, int n, cudaStream_t st);
void launch_tables_remove_hashed(const DevTables& T, const uint32_t* ids, const uint16_t* bkt,
                                 int64_t bkt_ld, int n, cudaStream_t st);

// ---------------------------------------------------------------------------
// Probe: per query the union of its L buckets with per-id counts, sorted by
// id, then the sampling strategy, the empty-set fallback and retain(id < N).
// ---------------------------------------------------------------------------
struct ProbeArgs {
  DevTables T;
  const uint16_t* bkt = nullptr;  // bucket of query s in table t: bkt[t*bkt_ld + s]
  int64_t bkt_ld = 0;
  int nq = 0;
  int N = 0;          // neuron count; 0 = plain index query (no selection)
  int sampling = KL_SAMPLING_VANILLA, top_k = 0, threshold = 0;
  int id_bits = 32;   // ids are < 2^id_bits
  uint32_t* out_ids = nullptr;
  uint32_t* out_counts = nullptr;  // nullable
  int out_stride = 0;              // capacity per query
  int32_t* out_n = nullptr;        // [nq] result sizes
  int* err = nullptr;
  unsigned long long* stat_active = nullptr;  // nullable: += sum of sizes
  int maxm = 0;       // set by launch_probe
  bool fallback = true;  // empty selection -> every neuron (layer.rs:82-84); off on a shard
  int mode = 0;       // set by launch_probe: 0 radix sort, 1 small-N count array, 2 bitmap (all selected)
};
// BOLT sparse inference over per-query candidate lists (ids sorted by id
// with their table counts, as the probe's COUNTS output).
struct BoltArgs {
  const uint32_t* cand_ids = nullptr;
  const uint32_t* cand_cnt = nullptr;
  const int32_t* cand_n = nullptr;
  int cand_stride = 0;
  int nq = 0, L = 0, k = 0, N = 0, d = 0;
  const float* X = nullptr;
  int64_t ldx = 0;
  const void* W = nullptr;
  int wdtype = 0;
  int64_t ldw = 0;
  const float* bias = nullptr;
  int relu = 1;
  uint32_t* out_ids = nullptr;
  float* out_act = nullptr;
  int32_t* out_n = nullptr;
  int out_stride = 0;
  int* err = nullptr;
  int maxm = 0, count_bits = 0;  // set by launch_bolt
};
void launch_bolt(const BoltArgs& a, cudaStream_t st);
size_t bolt_smem_bytes(int d, int cand_stride);
int probe_max_items();  // largest L*cap the probe kernel holds in shared memory
void launch_probe(const ProbeArgs& a, cudaStream_t st);

// Exclusive scan of n int32 counts into offsets[0..n] (offsets[n] = total).
size_t scan_scratch_bytes(int n);
void launch_scan(const int32_t* counts, int32_t* offsets, int n, void* scratch, cudaStream_t st);
// Compact per-query padded results into CSR (capacity-bounded).
void launch_compact(const uint32_t* ids, const uint32_t* counts, int stride, const int32_t* offs,
                    int nq, uint32_t* out_ids, uint32_t* out_counts, int32_t capacity,
                    int32_t* overflow, int* err, cudaStream_t st);

// ---------------------------------------------------------------------------
// Layer kernels (network/layer.rs, network/net.rs, optim/*.rs).
// ---------------------------------------------------------------------------
// Optimizer constants for one step, computed on the host exactly as the
// reference does in f32 (adam.rs:38-55: t = max(step,1), powi via
// square-and-multiply).
// Optimizer constants of one step.  The update kernels read them from device
// memory (written by the host before each train step), so a captured step
// graph stays valid as the step count changes.
struct OptStep {
  int opt;           // KL_OPT_*
  float lr, b1, b2, eps, omb1, omb2, c1, c2, mom;
};

// Active lists of one layer for a batch: ids[s*stride + a], a < cnt[s].
struct ActiveSet {
  uint32_t* ids;
  int32_t* cnt;
  int stride;
  float* pre;
  float* post;
  float* lg;
};

// Forward of a feature-major layer (W[d][ldw], neuron j of feature f at
// W[f*ldw + j]) over CSR input rows.  Writes pre/post and, if h != nullptr,
// the dense activation rows h[s*ldh + j] (h must be zeroed).
void launch_fm_forward(const void* W, int wdtype, int ldw, int d, const float* bias, int act,
                       SparseIn in, ActiveSet A, float* h, int ldh, int* err, cudaStream_t st);

// Row-major layer (W[N][ldw]) over dense inputs X[s*ldx + k], k < d.
enum RmMode { RM_FWD = 0, RM_FUSED = 1, RM_DX = 2 };
constexpr int RM_RPB = 256;  // active rows per block
struct RmArgs {
  const void* W;
  int wdtype, ldw, d;
  const float* bias;
  int act;
  const float* X;
  int ldx;
  ActiveSet A;
  float* h;           // FWD: dense output rows (nullable)
  int ldh;
  float* dxpart;      // FUSED/DX: [B][nchunk][ldx]
  int nchunk;
  const int32_t* lab_ptr;  // FUSED: label CSR (absolute offsets) and per-label activation
  const uint32_t* labels;
  float* labprob;
  int* err;
  uint32_t id_base;   // global id of local row 0 (neuron-sharded output layer; labels are global)
  const int32_t* only_empty;  // nullable: only examples s with only_empty[s] == 0 (the pass after a
                              // global empty-selection fallback); null: every example
  // FUSED, nullable: also store each local gradient into the dense update's
  // slot-major matrix, lgd_dense[slot_of[id] * ldb + s] (rows marked before the forward)
  float* lgd_dense;
  const uint32_t* slot_of;
  int64_t ldb;
};
void launch_rm_forward(const RmArgs& a, int nq, int mode, cudaStream_t st);
// dX[s][k] = sum over chunks of dxpart (chunk order).
void launch_reduce_dx(const float* dxpart, int nchunk, int ld, int d, const int32_t* cnt,
                      float* dx, int nq, cudaStream_t st);
// Softmax over each sample's active set (layer.rs:286-308); with labels, also
// the loss-gradient Jacobian product (layer.rs:141-176) into A.lg.
void launch_softmax(ActiveSet A, float* h, int ldh, const int32_t* lab_ptr,
                    const uint32_t* labels, float* labprob, int nq, cudaStream_t st);
// lg[s][a] = grad[s*ldg + id] * act'(pre, post) (layer.rs:177-193); softmax via
// the Jacobian.  If lgd != nullptr also the dense rows lgd[s*ldl + id] (zeroed
// by the caller) and the touched-neuron bitmask.
void launch_local_grads(ActiveSet A, int act, const float* grad, int ldg, float* lgd, int ldl,
                        uint32_t* touched_mask, int nq, cudaStream_t st);
// Per-sample loss (net.rs:180-199) from label activations, summed in sample
// order into *accum.
void launch_loss(const int32_t* lab_ptr, const float* labprob, int nq, float* accum,
                 cudaStream_t st);

// Row-major gradient + optimizer: rows touched by any active (s, a).
struct SegScratch {
  uint32_t* hist;     // [rows] zero between uses
  uint32_t* cur;      // [rows]
  uint32_t* touched;  // [rows]
  uint32_t* ctr;      // [4]: touched count, entry total, long-segment count (zeroed per use)
  uint32_t* ent_s;    // [entries]
  float* ent_v;       // [entries]
  uint32_t* slot;     // [rows] feature-major update: gradient row + 1 (0 = none), zero between uses
  uint32_t* longk;    // [rows] feature-major update: touched positions of long segments (count in ctr[2])
};
void launch_rm_update(const void* W, int wdtype, int ldw, int d, float* bias, float* m, float* v,
                      float* mb, float* vb, const float* X, int ldx, ActiveSet A, int nq, int N,
                      SegScratch S, const OptStep* o, unsigned long long* stat_touched,
                      cudaStream_t st);
// Dense-collision path of the row-major update: touched rows by mark words
// (first setter appends), local gradients scattered slot-major into LGd
// [round_up(rows, 32)][ldb] (all zero between steps), tiled bit-exact
// reduction.
struct DenseScratch {
  uint32_t* mark;      // [N] one word per row, zero between steps
  uint32_t* touched;   // [rows]
  uint32_t* slot_of;   // [N]
  uint32_t* ctr;       // [1] touched count (zeroed by the caller per step)
  float* LGd;          // [round_up(rows, 32)][ldb], zero between steps
  int64_t ldb;         // sample pitch: >= max batch, multiple of 32
};
bool rm_dense_fits(int64_t rows, int nb, int64_t max_bytes);
// stat += ctr[0] (touched-row counter of the roofline statistics)
void launch_count_touched(const uint32_t* ctr, unsigned long long* stat, cudaStream_t st);
// premarked: launch_rm_mark ran before the forward, which stored the
// gradients into D.LGd itself (mark and scatter are skipped here).
void launch_rm_update_dense(const void* W, int wdtype, int ldw, int d, float* bias, float* m, float* v,
                            float* mb, float* vb, const float* X, int ldx, ActiveSet A, int nq, int N,
                            DenseScratch D, const OptStep* o, unsigned long long* stat_touched,
                            cudaStream_t st, bool premarked = false);
// The dense update's row marking alone (touched list, slot_of), for a
// forward that stores its gradients straight into the matrix.
// only_empty (nullable): only examples s with only_empty[s] == 0.
void launch_rm_mark(ActiveSet A, int nq, DenseScratch D, cudaStream_t st, const int32_t* only_empty = nullptr);
// Feature-major gradient + optimizer over ALL features of the touched neurons
// (Adam decays every element of an active row, adam.rs:57-68).  G: gradient
// rows of the touched features, [min(d, nnz)][ldl] f32 scratch.  around_adam
// (nullable) is called with 0 before and 1 after the streaming Adam launch.
// S.slot must hold round_up(d, 4) + 4 entries (stages copy it in 16-byte units).
// Update of feature rows [f0, f0 + nf) of the feature-major layer (all d rows:
// f0 = 0, nf = d); the bias of every neuron is updated in every call.
void launch_fm_update(const void* W, int wdtype, int ldw, int d, int f0, int nf, int N, float* bias, float* m,
                      float* v, float* mb, float* vb, SparseIn in, const float* lgd, int ldl,
                      const uint32_t* touched_mask, SegScratch S, float* G, const OptStep* o,
                      unsigned long long* stat_touched, int* err, cudaStream_t st,
                      void (*around_adam)(void*, int) = nullptr, void* hook_arg = nullptr);

// Predict top-k over the final layer (net.rs:159-173): inactive neurons
// score 0; order by score descending, ties by lower id.
void launch_topk(ActiveSet A, int N, int k, uint32_t* top_ids, float* top_scores, int nq,
                 cudaStream_t st);

// Bit-exact f32/bf16 conversions of whole matrices (reference rows [n][d] <->
// device storage, optionally transposed for feature-major layers).
void launch_w_to_f32(const void* src, int wdtype, int64_t ld_src, bool transpose, float* dst,
                     int64_t n_rows, int d, cudaStream_t st);
void launch_f32_to_w(const float* src, int64_t n_rows, int d, int64_t ld_src, void* dst,
                     int wdtype, int64_t ld_dst, bool transpose, cudaStream_t st);


// ---------------------------------------------------------------------------
// Neuron-sharded train step (shard.cu).  A rank's batch is packed into a
// fixed layout of 32-bit words so that NCCL can all-gather equal-size blocks.
// ---------------------------------------------------------------------------
struct ShardLayout {
  int rowptr = 0, lptr = 0, idx = 0, val = 0, labels = 0, words = 0;  // word offsets / block size
};
ShardLayout shard_layout(int max_batch, int nnz_cap, int lab_cap);
void launch_shard_pack(uint32_t* send, const ShardLayout& Ly, const kl_batch& b, int B, uint32_t fault,
                       cudaStream_t st);
void launch_shard_unpack(const uint32_t* recv, const ShardLayout& Ly, int P, int B, int32_t* g_rowptr,
                         uint32_t* g_idx, float* g_val, int32_t* g_lptr, uint32_t* g_labels, int* err, OptStep* opt,
                         cudaStream_t st);
void launch_shard_fallback(ActiveSet A, const int32_t* gcnt, int n_local, int nq, int* err, cudaStream_t st);
// Global selection over the output shards (TopK below the candidate count,
// Threshold): per-example count histograms of the local candidates
// [nq][Lt + 1], the cut from the summed histograms, and the compaction of the
// local candidates into the active set (see shard.cu).
void launch_sel_hist(const uint32_t* ccnt, const int32_t* cn, int cstride, int Lt, int32_t* hist, int nq,
                     cudaStream_t st);
void launch_sel_cut(const int32_t* ghist, int Lt, int sampling, int top_k, int threshold, const uint32_t* ccnt,
                    const int32_t* cn, int cstride, int32_t* cut, int32_t* need, int32_t* gsel, int32_t* eqloc,
                    int nq, cudaStream_t st);
void launch_sel_apply(const uint32_t* cids, const uint32_t* ccnt, const int32_t* cn, int cstride, const int32_t* cut,
                      const int32_t* need, const int32_t* gsel, const int32_t* eq_all, int rank, int nq, int n_local,
                      ActiveSet A, int* err, unsigned long long* stat, cudaStream_t st);
// The global top k of this rank's B examples (global examples s0 ..) from
// every rank's local top-k lists ([P][PB][k] local ids and scores, P <= 64).
void launch_shard_topk_merge(const uint32_t* ids_all, const float* sc_all, int P, int PB, int k, int64_t N, int s0,
                             int B, uint32_t* top_ids, float* top_scores, cudaStream_t st);
void launch_shard_or_masks(uint32_t* tmask, const uint32_t* all, int P, int nw, cudaStream_t st);

// ---- Deja Vu sparse FFN (dejavu.cu) ----
// Rows per tcgen05 linear call (tokens); K pitch granularity of its weights.
constexpr int TC_LINEAR_MAX_T = 85;
constexpr int TC_LINEAR_KPAD = 64;
int tc_linear_splits(int n, int ldw, int* per, int ctas_per_sm);
size_t tc_linear_scratch_floats(int n, int ldw);
// y[T][n] = act(x[T][d] . W^T + bias), act 0 = ReLU, 1 = sigmoid; T <= 85;
// W [n][ldw] bf16 zero beyond d; xs scratch [3 * 85][ldw] bf16 holding the
// split x (x == nullptr: already written by the previous layer); P scratch of
// tc_linear_scratch_floats(n, ldw) floats; xs_next (nullable): y's pieces
// for a following layer of pitch ld_next.
void launch_tc_linear(const float* x, int T, int d, int ldx, const __nv_bfloat16* W, int n, int ldw,
                      const float* bias, int act, float* y, int ldy, __nv_bfloat16* xs, float* P,
                      __nv_bfloat16* xs_next, int ld_next, int* err, cudaStream_t st);
// The same y for T <= gemv_linear_max_tokens() tokens on the CUDA cores (one
// warp per weight row, f32 FMA sums); x [T][ldx] f32, no scratch.
int gemv_linear_max_tokens();
void launch_gemv_linear(const float* x, int T, int d, int ldx, const __nv_bfloat16* W, int n, int ldw,
                        const float* bias, int act, float* y, int ldy, cudaStream_t st);
// idx[t][0, k) = the k largest of scores[t][0, n) in (score desc, index asc)
// order; scores non-negative; k <= n.
// sorted: (score descending, index ascending); else the selected set in
// ascending index order (no sort)
void launch_topk(const float* scores, int T, int n, int lds, int k, uint32_t* idx, int ldi, cudaStream_t st,
                 bool sorted = true);
// out[T][hid] = SwiGLU MLP over the selected neurons sel[T][k]; gate/up
// [inter][ldw], downT [inter][ldw] bf16; a scratch [T][k], part scratch
// [T][splits][ldw] f32.
void launch_sparse_mlp(const __nv_bfloat16* gate, const __nv_bfloat16* up, const __nv_bfloat16* downT, int hid,
                       int ldw, int inter, const float* bias, const float* x, int T, const uint32_t* sel, int k,
                       float* a, float* part, int splits, float* out, bool accumulate, int* err,
                       cudaStream_t st);

// The same MLP as launch_sparse_mlp through dense tcgen05 GEMMs with the
// selection as a mask (T <= TC_LINEAR_MAX_T): gate / up [inter][ldg], down
// [hid][ldd] bf16 (ldg, ldd multiples of 64); scratch G, U [T][inter] f32,
// mask [T][inter] bytes (zero between calls), xs [3*85][ldg], hs [3*85][ldd]
// bf16, P of max(tc_linear_scratch_floats(inter, ldg), (hid, ldd)) floats.
void launch_sparse_mlp_dense(const __nv_bfloat16* gate, const __nv_bfloat16* up, const __nv_bfloat16* down,
                             int hid, int ldg, int inter, int ldd, const float* bias, const float* x, int T,
                             const uint32_t* sel, int k, float* G, float* U, uint8_t* mask, __nv_bfloat16* xs,
                             __nv_bfloat16* hs, float* P, float* out, int* err, cudaStream_t st);

// Deja Vu FFN stack helpers (dejavu.cu): RMSNorm of T rows of n and h += d.
void launch_rmsnorm(const float* x, int T, int n, const float* w, float eps, int one_plus, float* y,
                    cudaStream_t st);
void launch_residual_add(float* h, const float* d, int64_t n, cudaStream_t st);

void launch_set_opt(OptStep* dst, const OptStep& v, cudaStream_t st);

}  // namespace kl
