// pool_map.cu -- attention with a pooled attention map.
//
// Follows special_attentions/utils/attn_pooling_kernel.py (_attn_fwd_inner
// :25-97, _attention_pooling.forward :212-264): besides the attention output
// it returns Po[b, h, i, j] = max over the query rows r of block i of
// exp2(R[r, j] - m_r) / l_r, where R[r, j] is row r's largest logit (log2
// units, softmax scale folded in) in key block j and m_r, l_r are the row's
// final softmax max and sum; every row of Po is then divided by its sum.
//
// Here the block-sparse attention kernel records R (one fp32 per visited key
// block and row) and the row's log2-sum-exp lse_r = m_r + log2(l_r), so
// exp2(R - m) / l = exp2(R - lse); two small passes then reduce R over the
// rows of each query block and normalise the rows of Po.  Key blocks a row
// does not visit (sparse block lists) contribute 0.
#include "saf_common.cuh"

int32_t bsa_fwd_entry(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                      const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                      int64_t col_capacity, int32_t block_m, int32_t block_n, const float* kv_bias,
                      int64_t kv_bias_stride_bh, float sm_scale, int32_t lead_rows,
                      const int32_t* row_ranges, const saf::FrameMaskArgs* frames, float* pool_rmax,
                      float* pool_lse, void* stream);

namespace saf {
namespace {

__global__ void __launch_bounds__(256) fill_kernel(float* x, int64_t n, float v) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    x[i] = v;
}

// One warp per (head, key block j); the lanes walk the query rows of every
// query block i (coalesced along the rows).  A row with lse = -inf (no
// visible key) contributes 0.
__global__ void __launch_bounds__(256) pool_map_kernel(const float* __restrict__ rmax,
                                                       const float* __restrict__ lse, int BH, int nbk,
                                                       int Sq, int pb, int nbp, float* __restrict__ po) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= static_cast<int64_t>(BH) * nbk) return;
  const int g = static_cast<int>(w / nbk), j = static_cast<int>(w % nbk);
  const float* R = rmax + (static_cast<int64_t>(g) * nbk + j) * Sq;
  const float* L = lse + static_cast<int64_t>(g) * Sq;
  for (int i = 0; i < nbp; ++i) {
    const int r0 = i * pb, r1 = min(r0 + pb, Sq);
    float m = 0.f;
    for (int r = r0 + lane; r < r1; r += 32) {
      const float l = L[r];
      m = fmaxf(m, l == -INFINITY ? 0.f : exp2f(R[r] - l));
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) po[(static_cast<int64_t>(g) * nbp + i) * nbk + j] = m;
  }
}

// One warp per row of Po: divide by the row sum (lane l sums columns l,
// l + 32, ... ascending, then an xor butterfly).  An all-zero row gives NaN,
// as the reference's division.
__global__ void __launch_bounds__(256) pool_norm_kernel(float* __restrict__ po, int64_t rows, int nbk) {
  const int64_t w = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (w >= rows) return;
  float* row = po + w * nbk;
  float s = 0.f;
  for (int j = lane; j < nbk; j += 32) s += row[j];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  for (int j = lane; j < nbk; j += 32) row[j] = row[j] / s;
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" int64_t saf_bsa_pool_workspace_bytes(int64_t BH, int64_t Sq, int32_t nbk) {
  if (BH <= 0 || Sq <= 0 || nbk <= 0) return 0;
  return 4 * BH * Sq * (static_cast<int64_t>(nbk) + 1) + 256;
}

extern "C" int32_t saf_bsa_fwd_pool(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                                    const saf_tensor4* o, const int32_t* row_ptr,
                                    const int32_t* col_idx, int64_t col_capacity, int32_t block_m,
                                    int32_t block_n, float sm_scale, int32_t lead_rows,
                                    int32_t pool_block, void* workspace, int64_t workspace_bytes,
                                    float* pool_out, void* stream) {
  int32_t rc = check_tensor4(q);
  if (rc != SAF_OK) return rc;
  if (k == nullptr || check_tensor4(k) != SAF_OK) return SAF_ERR_ARG;
  if (q->dtype != SAF_BF16 && q->dtype != SAF_F16) return SAF_ERR_UNSUPPORTED;
  if (pool_block <= 0 || block_n <= 0 || pool_out == nullptr || workspace == nullptr) return SAF_ERR_ARG;
  const int64_t BH = q->B * q->H, Sq = q->S;
  const int64_t nbk = (k->S + block_n - 1) / block_n;
  const int64_t nbp = (Sq + pool_block - 1) / pool_block;
  if (nbk > 0x7fffffff || Sq > 0x7fffffff) return SAF_ERR_SHAPE;
  if (workspace_bytes < saf_bsa_pool_workspace_bytes(BH, Sq, static_cast<int32_t>(nbk))) return SAF_ERR_ARG;
  float* rmax = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  float* lse = rmax + BH * nbk * Sq;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
  const int64_t n_r = BH * nbk * Sq;
  fill_kernel<<<static_cast<unsigned>(std::min<int64_t>((n_r + 255) / 256, 148 * 32)), 256, 0, st>>>(
      rmax, n_r, -INFINITY);
  SAF_CUDA_TRY(cudaGetLastError());
  rc = bsa_fwd_entry(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, nullptr, 0, sm_scale,
                     lead_rows, nullptr, nullptr, rmax, lse, stream);
  if (rc != SAF_OK) return rc;
  const int64_t warps1 = BH * nbk, warps2 = BH * nbp;
  pool_map_kernel<<<static_cast<unsigned>((warps1 + 7) / 8), 256, 0, st>>>(
      rmax, lse, static_cast<int>(BH), static_cast<int>(nbk), static_cast<int>(Sq), pool_block,
      static_cast<int>(nbp), pool_out);
  SAF_CUDA_TRY(cudaGetLastError());
  pool_norm_kernel<<<static_cast<unsigned>((warps2 + 7) / 8), 256, 0, st>>>(pool_out, warps2,
                                                                           static_cast<int>(nbk));
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
