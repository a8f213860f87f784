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
  shard_header_kernel<<<1, 256, 0, st>>>(send, B, fault ? 0 : b.nnz, fault ? 0 : b.nlabels, fault, rp, lp);
  count_launch();
  if (fault) return;
  cudaMemcpyAsync(rp, b.rowptr, (size_t)(B + 1) * 4, cudaMemcpyDeviceToDevice, st);
  cudaMemcpyAsync(lp, b.label_ptr, (size_t)(B + 1) * 4, cudaMemcpyDeviceToDevice, st);
  if (b.nnz > 0) {
    cudaMemcpyAsync(send + Ly.idx, b.idx, (size_t)b.nnz * 4, cudaMemcpyDeviceToDevice, st);
    cudaMemcpyAsync(send + Ly.val, b.val, (size_t)b.nnz * 4, cudaMemcpyDeviceToDevice, st);
  }
  if (b.nlabels > 0) cudaMemcpyAsync(send + Ly.labels, b.labels, (size_t)b.nlabels * 4, cudaMemcpyDeviceToDevice, st);
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
