// shard.cu -- kernels of the neuron-sharded train step (one process per GPU).
//
// The output layer's neurons are split into P contiguous slices, one per
// rank; the sparse-input hidden layer is data parallel: rank r holds examples
// [r*B, (r+1)*B) of the global batch of P*B examples (rank-major order).
// These kernels move the per-rank batches in and out of the fixed-size word
// buffers that NCCL all-gathers, and apply the decisions that must be made
// over all shards.
#include "engine.h"

namespace kl {
namespace {

// Header of a packed batch: B, nnz, nlabels and a fault word.  A rank whose
// batch cannot be exchanged (wrong example count, or more nnz / labels than
// the fixed exchange capacity) sends an empty batch of B examples with the
// fault word set (a DERR_* bit) instead of leaving the collective sequence,
// so every rank stays in step and every rank sees the fault.
__global__ void shard_header_kernel(uint32_t* send, int B, int nnz, int nlab, uint32_t fault, int32_t* rowptr_empty,
                                    int32_t* lptr_empty) {
  if (threadIdx.x == 0) {
    send[0] = (uint32_t)B;
    send[1] = (uint32_t)nnz;
    send[2] = (uint32_t)nlab;
    send[3] = fault;
  }
  if (fault)
    for (int s = threadIdx.x; s <= B; s += blockDim.x) {
      rowptr_empty[s] = 0;
      lptr_empty[s] = 0;
    }
}

// Block r rebuilds rank r's part of the global batch from the gathered
// buffers: CSR rows and label rows are appended in rank order with their
// offsets rebased onto the global arrays.
// A fault word from any rank is raised on every rank, and the step's learning
// rate is set to 0 so that no weight moves (Adam moments still advance).
__global__ void shard_unpack_kernel(const uint32_t* recv, ShardLayout Ly, int P, int B, int32_t* g_rowptr,
                                    uint32_t* g_idx, float* g_val, int32_t* g_lptr, uint32_t* g_labels, int* err,
                                    OptStep* opt) {
  const int r = blockIdx.x;
  __shared__ uint32_t pre_nnz, pre_lab;
  if (threadIdx.x == 0) {
    uint32_t a = 0, b = 0;
    for (int q = 0; q < r; ++q) {
      a += recv[(size_t)q * Ly.words + 1];
      b += recv[(size_t)q * Ly.words + 2];
    }
    pre_nnz = a;
    pre_lab = b;
    uint32_t fault = 0;
    for (int q = 0; q < P; ++q) {
      if ((int)recv[(size_t)q * Ly.words] != B) fault |= DERR_BOUNDS;  // every rank must pass B examples
      fault |= recv[(size_t)q * Ly.words + 3];
    }
    if (fault) {
      atomicOr(err, (int)fault);
      if (r == 0) opt->lr = 0.0f;
    }
  }
  __syncthreads();
  const uint32_t* blk = recv + (size_t)r * Ly.words;
  const int nnz = (int)blk[1], nlab = (int)blk[2];
  const int32_t* rp = reinterpret_cast<const int32_t*>(blk + Ly.rowptr);
  const int32_t* lp = reinterpret_cast<const int32_t*>(blk + Ly.lptr);
  const int32_t rp0 = rp[0], lp0 = lp[0];
  for (int s = threadIdx.x; s < B; s += blockDim.x) {
    g_rowptr[(int64_t)r * B + s] = (int32_t)pre_nnz + (rp[s] - rp0);
    g_lptr[(int64_t)r * B + s] = (int32_t)pre_lab + (lp[s] - lp0);
  }
  if (r == P - 1 && threadIdx.x == 0) {
    g_rowptr[(int64_t)P * B] = (int32_t)(pre_nnz + nnz);
    g_lptr[(int64_t)P * B] = (int32_t)(pre_lab + nlab);
  }
  for (int e = threadIdx.x; e < nnz; e += blockDim.x) {
    g_idx[pre_nnz + e] = blk[Ly.idx + e];
    g_val[pre_nnz + e] = __uint_as_float(blk[Ly.val + e]);
  }
  for (int e = threadIdx.x; e < nlab; e += blockDim.x) g_labels[pre_lab + e] = blk[Ly.labels + e];
}

// Global empty-selection fallback (layer.rs:82-84) on a shard: a sample whose
// selection is empty on EVERY shard takes all neurons, so this shard takes
// all of its own.
__global__ void shard_fallback_kernel(ActiveSet A, const int32_t* gcnt, int n_local, int nq, int* err) {
  const int s = blockIdx.x;
  if (s >= nq || gcnt[s] != 0) return;
  const int n = min(n_local, A.stride);
  if (n_local > A.stride && threadIdx.x == 0) atomicOr(err, DERR_CAPACITY);
  for (int j = threadIdx.x; j < n; j += blockDim.x) A.ids[(int64_t)s * A.stride + j] = (uint32_t)j;
  if (threadIdx.x == 0) A.cnt[s] = n;
}

// ---- global selection over the shards (TopK below the candidate count,
// Threshold).  The reference selects over the whole layer's candidates
// (topk.rs:19-34: count descending, then id ascending; threshold.rs:20-43:
// every count >= threshold, else the single best).  Each rank probes its
// slice for every candidate with its table count; the ranks then agree on
// a per-example cut from the summed count histograms: every candidate with
// count > cut is taken, plus the `need` lowest-id candidates with count ==
// cut, which lie on the lowest ranks first (slices are contiguous in id).
constexpr int SEL_NT = 256;

// hist[s][c] = #local candidates of example s with table count c (c <= Lt)
__global__ void sel_hist_kernel(const uint32_t* ccnt, const int32_t* cn, int cstride, int Lt, int32_t* hist) {
  extern __shared__ int32_t h[];
  const int s = blockIdx.x;
  for (int c = threadIdx.x; c <= Lt; c += SEL_NT) h[c] = 0;
  __syncthreads();
  const int n = cn[s];
  for (int u = threadIdx.x; u < n; u += SEL_NT)
    atomicAdd(&h[min((int)ccnt[(int64_t)s * cstride + u], Lt)], 1);
  __syncthreads();
  for (int c = threadIdx.x; c <= Lt; c += SEL_NT) hist[(int64_t)s * (Lt + 1) + c] = h[c];
}

// From the global histogram: cut, need and the global selection size of
// example s, and this rank's number of candidates with count == cut.
__global__ void sel_cut_kernel(const int32_t* ghist, int Lt, int sampling, int top_k, int threshold,
                               const uint32_t* ccnt, const int32_t* cn, int cstride, int32_t* cut_o,
                               int32_t* need_o, int32_t* gsel_o, int32_t* eqloc_o) {
  __shared__ int cut_s, tmp[33];
  const int s = blockIdx.x;
  if (threadIdx.x == 0) {
    const int32_t* h = ghist + (int64_t)s * (Lt + 1);
    int cut = 0, need = 0, gsel = 0;
    if (sampling == KL_SAMPLING_TOPK) {
      int total = 0;
      for (int c = 1; c <= Lt; ++c) total += h[c];
      if (total <= top_k) {
        gsel = total;  // every candidate
      } else {
        int acc = 0;
        for (int c = Lt; c >= 1; --c) {
          if (acc + h[c] >= top_k) {
            cut = c;
            need = top_k - acc;
            break;
          }
          acc += h[c];
        }
        gsel = top_k;
      }
    } else {  // KL_SAMPLING_THRESHOLD
      const int thr = max(threshold, 1);
      int pass = 0, cmax = 0;
      for (int c = 1; c <= Lt; ++c) {
        if (c >= thr) pass += h[c];
        if (h[c] > 0) cmax = c;
      }
      if (pass > 0) {
        cut = thr - 1;
        gsel = pass;
      } else if (cmax > 0) {
        cut = cmax;  // the single best: the lowest id among the highest count
        need = 1;
        gsel = 1;
      } else {
        cut = Lt + 1;  // no candidate anywhere
      }
    }
    cut_o[s] = cut;
    need_o[s] = need;
    gsel_o[s] = gsel;
    cut_s = need > 0 ? cut : -1;
  }
  __syncthreads();
  const int cut = cut_s;
  int eq = 0;
  if (cut >= 0)
    for (int u = threadIdx.x; u < cn[s]; u += SEL_NT) eq += (int)ccnt[(int64_t)s * cstride + u] == cut;
  eq = block_sum<SEL_NT>(eq, tmp);
  if (threadIdx.x == 0) eqloc_o[s] = eq;
}

// The selection of example s on this rank, in id order, into the active set;
// an example that no rank selects anything for takes every local neuron.
__global__ void sel_apply_kernel(const uint32_t* cids, const uint32_t* ccnt, const int32_t* cn, int cstride,
                                 const int32_t* cut_a, const int32_t* need_a, const int32_t* gsel_a,
                                 const int32_t* eq_all, int rank, int nq, int n_local, ActiveSet A, int* err,
                                 unsigned long long* stat) {
  __shared__ int tmp[33];
  const int s = blockIdx.x;
  uint32_t* out = A.ids + (int64_t)s * A.stride;
  if (gsel_a[s] == 0) {  // fallback (layer.rs:82-84) over the global selection
    const int n = min(n_local, A.stride);
    if (n_local > A.stride && threadIdx.x == 0) atomicOr(err, DERR_CAPACITY);
    for (int j = threadIdx.x; j < n; j += SEL_NT) out[j] = (uint32_t)j;
    if (threadIdx.x == 0) {
      A.cnt[s] = n;
      if (stat) atomicAdd(stat, (unsigned long long)n);
    }
    return;
  }
  const int cut = cut_a[s];
  int take = 0;
  if (need_a[s] > 0) {
    int before = 0;  // candidates with count == cut on lower ranks (lower ids)
    for (int q = 0; q < rank; ++q) before += eq_all[(int64_t)q * nq + s];
    take = max(0, need_a[s] - before);
  }
  const int n = cn[s];
  const uint32_t* ci = cids + (int64_t)s * cstride;
  const uint32_t* cc = ccnt + (int64_t)s * cstride;
  // blocked arrangement keeps id order: thread t owns candidates [t*UPT, (t+1)*UPT)
  const int UPT = (n + SEL_NT - 1) / SEL_NT;
  const int u0 = threadIdx.x * UPT, u1 = min(n, u0 + UPT);
  int eq = 0;
  for (int u = u0; u < u1; ++u) eq += (int)cc[u] == cut;
  int eq_tot;
  int eq_rank = block_excl_scan<SEL_NT>(eq, tmp, &eq_tot);
  int keep = 0;
  {
    int r = eq_rank;
    for (int u = u0; u < u1; ++u) {
      const int c = (int)cc[u];
      keep += c > cut || (c == cut && r++ < take);
    }
  }
  int nsel;
  int pos = block_excl_scan<SEL_NT>(keep, tmp, &nsel);
  for (int u = u0; u < u1; ++u) {
    const int c = (int)cc[u];
    const bool k = c > cut || (c == cut && eq_rank++ < take);
    if (k) {
      if (pos < A.stride) out[pos] = ci[u];
      ++pos;
    }
  }
  if (threadIdx.x == 0) {
    if (nsel > A.stride) atomicOr(err, DERR_CAPACITY);
    A.cnt[s] = min(nsel, A.stride);
    if (stat) atomicAdd(stat, (unsigned long long)min(nsel, A.stride));
  }
}

// predict_top_k over the shards: rank q's list for example s is its slice's
// top k in (score descending, id ascending) order with local ids; the global
// top k of this rank's example i (global example s0 + i) is a P-way merge of
// those lists in the same order on global ids (slice q starts at q*N/P).
__global__ void shard_topk_merge_kernel(const uint32_t* ids_all, const float* sc_all, int P, int PB, int k,
                                        int64_t N, int s0, int B, uint32_t* top_ids, float* top_scores) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= B) return;
  const int s = s0 + i;
  constexpr int PMAX = 64;
  int pos[PMAX];
  for (int q = 0; q < P; ++q) pos[q] = 0;
  for (int o = 0; o < k; ++o) {
    int best = -1;
    float bs = 0.0f;
    uint32_t bid = 0;
    for (int q = 0; q < P; ++q) {
      if (pos[q] >= k) continue;
      const int64_t e = ((int64_t)q * PB + s) * k + pos[q];
      const float v = sc_all[e];
      const uint32_t g = ids_all[e] + (uint32_t)(((int64_t)q * N) / P);
      if (best < 0 || v > bs || (v == bs && g < bid)) {
        best = q;
        bs = v;
        bid = g;
      }
    }
    ++pos[best];
    top_ids[(int64_t)i * k + o] = bid;
    if (top_scores) top_scores[(int64_t)i * k + o] = bs;
  }
}

__global__ void shard_or_masks_kernel(uint32_t* tmask, const uint32_t* all, int P, int nw) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nw) return;
  uint32_t v = 0;
  for (int q = 0; q < P; ++q) v |= all[(size_t)q * nw + i];
  tmask[i] = v;
}

}  // namespace

ShardLayout shard_layout(int max_batch, int nnz_cap, int lab_cap) {
  ShardLayout L;
  L.rowptr = 4;
  L.lptr = L.rowptr + max_batch + 1;
  L.idx = L.lptr + max_batch + 1;
  L.val = L.idx + nnz_cap;
  L.labels = L.val + nnz_cap;
  L.words = (int)round_up(L.labels + lab_cap, 32);
  return L;
}

void launch_shard_pack(uint32_t* send, const ShardLayout& Ly, const kl_batch& b, int B, uint32_t fault,
                       cudaStream_t st) {
  int32_t* rp = reinterpret_cast<int32_t*>(send + Ly.rowptr);
  int32_t* lp = reinterpret_cast<int32_t*>(send + Ly.lptr);
  // a batch without labels (inference) travels with empty label rows
  const int nlab = b.label_ptr ? b.nlabels : 0;
  shard_header_kernel<<<1, 256, 0, st>>>(send, B, fault ? 0 : b.nnz, fault ? 0 : nlab, fault, rp, lp);
  count_launch();
  if (fault) return;
  cudaMemcpyAsync(rp, b.rowptr, (size_t)(B + 1) * 4, cudaMemcpyDeviceToDevice, st);
  if (b.label_ptr) cudaMemcpyAsync(lp, b.label_ptr, (size_t)(B + 1) * 4, cudaMemcpyDeviceToDevice, st);
  else cudaMemsetAsync(lp, 0, (size_t)(B + 1) * 4, st);
  if (b.nnz > 0) {
    cudaMemcpyAsync(send + Ly.idx, b.idx, (size_t)b.nnz * 4, cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(send + Ly.val, b.val, (size_t)b.nnz * 4, cudaMemcpyDeviceToDevice, st);
  }
  if (nlab > 0) cudaMemcpyAsync(send + Ly.labels, b.labels, (size_t)nlab * 4, cudaMemcpyDeviceToDevice, st);
}

void launch_shard_unpack(const uint32_t* recv, const ShardLayout& Ly, int P, int B, int32_t* g_rowptr,
                         uint32_t* g_idx, float* g_val, int32_t* g_lptr, uint32_t* g_labels, int* err, OptStep* opt,
                         cudaStream_t st) {
  shard_unpack_kernel<<<P, 512, 0, st>>>(recv, Ly, P, B, g_rowptr, g_idx, g_val, g_lptr, g_labels, err, opt);
  count_launch();
}

void launch_shard_fallback(ActiveSet A, const int32_t* gcnt, int n_local, int nq, int* err, cudaStream_t st) {
  if (nq <= 0) return;
  shard_fallback_kernel<<<nq, 256, 0, st>>>(A, gcnt, n_local, nq, err);
  count_launch();
}

void launch_sel_hist(const uint32_t* ccnt, const int32_t* cn, int cstride, int Lt, int32_t* hist, int nq,
                     cudaStream_t st) {
  if (nq <= 0) return;
  sel_hist_kernel<<<nq, SEL_NT, (size_t)(Lt + 1) * 4, st>>>(ccnt, cn, cstride, Lt, hist);
  count_launch();
}
void launch_sel_cut(const int32_t* ghist, int Lt, int sampling, int top_k, int threshold, const uint32_t* ccnt,
                    const int32_t* cn, int cstride, int32_t* cut, int32_t* need, int32_t* gsel, int32_t* eqloc,
                    int nq, cudaStream_t st) {
  if (nq <= 0) return;
  sel_cut_kernel<<<nq, SEL_NT, 0, st>>>(ghist, Lt, sampling, top_k, threshold, ccnt, cn, cstride, cut, need, gsel,
                                        eqloc);
  count_launch();
}
void launch_sel_apply(const uint32_t* cids, const uint32_t* ccnt, const int32_t* cn, int cstride, const int32_t* cut,
                      const int32_t* need, const int32_t* gsel, const int32_t* eq_all, int rank, int nq, int n_local,
                      ActiveSet A, int* err, unsigned long long* stat, cudaStream_t st) {
  if (nq <= 0) return;
  sel_apply_kernel<<<nq, SEL_NT, 0, st>>>(cids, ccnt, cn, cstride, cut, need, gsel, eq_all, rank, nq, n_local, A,
                                          err, stat);
  count_launch();
}

void launch_shard_topk_merge(const uint32_t* ids_all, const float* sc_all, int P, int PB, int k, int64_t N, int s0,
                             int B, uint32_t* top_ids, float* top_scores, cudaStream_t st) {
  if (B <= 0 || k <= 0) return;
  shard_topk_merge_kernel<<<(unsigned)ceil_div(B, 128), 128, 0, st>>>(ids_all, sc_all, P, PB, k, N, s0, B, top_ids,
                                                                     top_scores);
  count_launch();
}

void launch_shard_or_masks(uint32_t* tmask, const uint32_t* all, int P, int nw, cudaStream_t st) {
  shard_or_masks_kernel<<<(unsigned)ceil_div(nw, 256), 256, 0, st>>>(tmask, all, P, nw);
  count_launch();
}

namespace {
__global__ void flag_error_kernel(int* err, int bits) { atomicOr(err, bits); }
__global__ void set_opt_kernel(OptStep* dst, OptStep v) { *dst = v; }
}  // namespace
// The step's optimizer constants travel as a kernel argument: a copy from
// pageable host memory could make the host wait for the stream.
void launch_set_opt(OptStep* dst, const OptStep& v, cudaStream_t st) {
  set_opt_kernel<<<1, 1, 0, st>>>(dst, v);
  count_launch();
}
void flag_error(int* err, int bits, cudaStream_t st) {
  flag_error_kernel<<<1, 1, 0, st>>>(err, bits);
  count_launch();
}

}  // namespace kl
