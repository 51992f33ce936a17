// pool_map.cu -- attention with a pooled attention map.
//
// Follows special_attentions/utils/attn_pooling_kernel.py (_attn_fwd_inner
// :25-97, _attention_pooling.forward :212-264): besides the attention output
// it returns Po[b, h, i, j] = max over the query rows r of pool block i of
// exp2(R[r, j] - m_r) / l_r, where R[r, j] is row r's largest logit (log2
// units, softmax scale folded in) in key block j and m_r, l_r are the row's
// final softmax max and sum; every row of Po is then divided by its sum.
//
// The block-sparse attention kernel does all of it: per visited key block
// the softmax warps keep each row's R in a per-CTA scratch slot (the tile's
// parity; it stays in L2) and, at the tile's end, its log2-sum-exp
// lse_r = m_r + log2(l_r) in shared memory; the CTA's otherwise idle warps
// 2-3 then reduce exp2(R - lse) over the rows of each pool block and pool
// them into the map by an atomic max, while the softmax warps go on with
// the next tile.  A small pass divides every pooled row by its sum.  Key
// blocks a row does not visit (sparse block lists) contribute 0: the map is
// zeroed first.
#include "saf_common.cuh"

int32_t bsa_fwd_entry(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                      const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                      int64_t col_capacity, int32_t block_m, int32_t block_n, const float* kv_bias,
                      int64_t kv_bias_stride_bh, float sm_scale, int32_t lead_rows,
                      const int32_t* row_ranges, const saf::FrameMaskArgs* frames, const saf::PoolArgs* pool,
                      void* stream);

namespace saf {
namespace {

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

// Scratch: every persistent CTA (at most two per SM) keeps 128 rows x the
// key blocks of its last two tiles (one being written, one being pooled).
extern "C" int64_t saf_bsa_pool_workspace_bytes(int64_t BH, int64_t Sq, int32_t nbk) {
  if (BH <= 0 || Sq <= 0 || nbk <= 0) return 0;
  int dev = 0, sms = 0;
  if (cudaGetDevice(&dev) != cudaSuccess ||
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    sms = 256;  // no device here: an upper bound for any sm_100 part
  const int64_t cap = (static_cast<int64_t>(nbk) + 7) / 8 * 8;
  return 2 * static_cast<int64_t>(sms) * 2 * cap * 128 * 4 + 256;  // CTAs x two tile slots
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
  if (block_n <= 0 || pool_out == nullptr || workspace == nullptr) return SAF_ERR_ARG;
  // a pooled row is one 128-row tile or one half of it
  if (pool_block != 64 && pool_block != 128) return SAF_ERR_UNSUPPORTED;
  if (block_m == 128 && pool_block != 128) return SAF_ERR_UNSUPPORTED;
  const int64_t BH = q->B * q->H, Sq = q->S;
  const int64_t nbk = (k->S + block_n - 1) / block_n;
  const int64_t nbp = (Sq + pool_block - 1) / pool_block;
  if (nbk > 0x7fffffff || Sq > 0x7fffffff) return SAF_ERR_SHAPE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
  if (workspace_bytes < saf_bsa_pool_workspace_bytes(BH, Sq, static_cast<int32_t>(nbk))) return SAF_ERR_ARG;
  float* scratch = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  SAF_CUDA_TRY(cudaMemsetAsync(pool_out, 0, static_cast<size_t>(BH * nbp * nbk) * sizeof(float), st));
  const PoolArgs pa{scratch, pool_out, pool_block};
  rc = bsa_fwd_entry(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, nullptr, 0, sm_scale,
                     lead_rows, nullptr, nullptr, &pa, stream);
  if (rc != SAF_OK) return rc;
  const int64_t rows = BH * nbp;
  pool_norm_kernel<<<static_cast<unsigned>((rows + 7) / 8), 256, 0, st>>>(pool_out, rows, static_cast<int>(nbk));
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
