// bsa_simt.cu -- block-sparse attention in full fp32 on the CUDA cores, and
// the saf_bsa_fwd entry point that validates arguments and dispatches by
// element type (16-bit -> tcgen05 kernel in bsa_sm100.cu, fp32 -> here).
//
// The fp32 path exists because the fp32 configuration is checked to 1e-4,
// which rules out TF32 tensor-core products.  Same semantics as the
// reference kernel (special_attentions/utils/block_sparse_attn_kernel.py:
// 52-209): online softmax with natural exp, keys past seqlen_k masked,
// zero row sum -> NaN.  Mask blocks must be multiples of 64 rows/columns;
// the CTA computes 64 x 64 sub-tiles.
#include "saf_common.cuh"

namespace saf {

int32_t bsa_fwd_sm100(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                      const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                      int64_t col_capacity, int bm, int bn, const float* kv_bias,
                      int64_t bias_stride, float sm_scale, int lead_tiles, const int32_t* row_ranges,
                      const FrameMaskArgs* frames, const PoolArgs* pool,
                      cudaStream_t stream);
int32_t bsa_fwd_sm100_keys(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                           const saf_tensor4* o, const int32_t* key_list, int32_t key_len,
                           const int32_t* key_batch, float sm_scale, cudaStream_t stream);

namespace {

constexpr int kT = 64;  // sub-tile edge

struct SimtParams {
  const float* q;
  const float* k;
  const float* v;
  float* o;
  int H, Sq, Sk;
  int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss, v_sb, v_sh, v_ss, o_sb, o_sh, o_ss;
  int bm, bn, nbq, nbk;
  int64_t col_capacity;
  const int32_t* row_ptr;
  const int32_t* col_idx;
  const float* kv_bias;
  int64_t bias_stride;
  float scale;
  unsigned int* status;
  const int4* row_ranges;  // nullable [Sq]: key intervals [x, y) U [z, w) of each query row
};

// grid (ceil(Sq/64), B*H), 256 threads.  Thread (ty, tx) in a 16 x 16 grid
// owns S rows ty*4..+3, columns tx*4..+3, and O rows ty*4..+3,
// columns tx*(D/16)..+D/16.
template <int D>
__global__ void __launch_bounds__(256) bsa_fwd_simt_kernel(const SimtParams p) {
  constexpr int DC = D / 16;  // O columns per thread
  extern __shared__ float sm[];
  float* qt = sm;                // [D][64]  (q transposed)
  float* kt = qt + D * kT;       // [D][64]  (k transposed)
  float* vs = kt + D * kT;       // [64][D]
  float* ss = vs + kT * D;       // [64][65] scores / probabilities
  float* alpha_s = ss + kT * (kT + 1);  // [64]
  float* bias_s = alpha_s + kT;         // [64]

  const int tile = blockIdx.x, g = blockIdx.y;
  const int b = g / p.H, h = g % p.H;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int q0 = tile * kT;
  const float* qg = p.q + b * p.q_sb + h * p.q_sh;
  const float* kg = p.k + b * p.k_sb + h * p.k_sh;
  const float* vg = p.v + b * p.v_sb + h * p.v_sh;

  for (int idx = tid; idx < kT * D; idx += 256) {
    const int r = idx / D, d = idx % D;
    const int row = q0 + r;
    qt[d * kT + r] = row < p.Sq ? qg[static_cast<int64_t>(row) * p.q_ss + d] : 0.f;
  }

  float acc[4][DC];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < DC; ++c) acc[i][c] = 0.f;
  // running max / sum of row (ty*4 + i); kept redundantly by the 16 threads
  // of a row group (each computes the same values from shared memory).
  float m_run[4], l_run[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m_run[i] = -INFINITY;
    l_run[i] = 0.f;
  }

  const int mrow = q0 / p.bm;
  const int32_t* rp = p.row_ptr + static_cast<int64_t>(g) * (p.nbq + 1);
  auto clampi = [&](int64_t x) {
    return x < 0 ? int64_t(0) : (x > p.col_capacity ? p.col_capacity : x);
  };
  const int64_t e_beg = clampi(rp[mrow]), e_end = clampi(rp[mrow + 1]);
  const int subs = p.bn / kT;
  for (int64_t e = e_beg; e < e_end; ++e) {
    const int col = p.col_idx[e];
    if (col < 0 || col >= p.nbk) {
      if (tid == 0) atomicOr(p.status, SAF_DEV_BADINDEX);
      continue;
    }
    for (int u = 0; u < subs; ++u) {
      const int k0 = col * p.bn + u * kT;
      if (k0 >= p.Sk) break;
      __syncthreads();  // previous tile fully consumed
      for (int idx = tid; idx < kT * D; idx += 256) {
        const int r = idx / D, d = idx % D;
        const int row = k0 + r;
        kt[d * kT + r] = row < p.Sk ? kg[static_cast<int64_t>(row) * p.k_ss + d] : 0.f;
        vs[r * D + d] = row < p.Sk ? vg[static_cast<int64_t>(row) * p.v_ss + d] : 0.f;
      }
      if (tid < kT) {
        const int row = k0 + tid;
        bias_s[tid] = (p.kv_bias != nullptr && row < p.Sk)
                          ? p.kv_bias[static_cast<int64_t>(g) * p.bias_stride + row]
                          : 0.f;
      }
      __syncthreads();
      // S = scale * Q K^T + bias, masked past Sk.
      float s[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
      for (int d = 0; d < D; ++d) {
        const float4 a = *reinterpret_cast<const float4*>(&qt[d * kT + ty * 4]);
        const float4 bb = *reinterpret_cast<const float4*>(&kt[d * kT + tx * 4]);
        const float av[4] = {a.x, a.y, a.z, a.w}, bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 4; ++c) s[i][c] = fmaf(av[i], bv[c], s[i][c]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int kc = tx * 4 + c;
          bool keep = k0 + kc < p.Sk;
          if (p.row_ranges != nullptr) {
            const int qr = q0 + ty * 4 + i, kk = k0 + kc;
            if (qr < p.Sq) {
              const int4 rr = __ldg(p.row_ranges + qr);
              keep = keep && ((kk >= rr.x && kk < rr.y) || (kk >= rr.z && kk < rr.w));
            }
          }
          ss[(ty * 4 + i) * (kT + 1) + kc] = keep ? s[i][c] * p.scale + bias_s[kc] : -INFINITY;
        }
      __syncthreads();
      // Row softmax update: the 16 threads of row group ty split the columns.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty * 4 + i;
        float mx = -INFINITY;
        for (int c = tx; c < kT; c += 16) mx = fmaxf(mx, ss[r * (kT + 1) + c]);
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        const float m_new = fmaxf(m_run[i], mx);
        const float m_safe = (m_new == -INFINITY) ? 0.f : m_new;
        const float alpha = expf(m_run[i] - m_safe);
        float sum = 0.f;
        for (int c = tx; c < kT; c += 16) {
          const float pv = expf(ss[r * (kT + 1) + c] - m_safe);
          ss[r * (kT + 1) + c] = pv;
          sum += pv;
        }
#pragma unroll
        for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
        l_run[i] = l_run[i] * alpha + sum;
        m_run[i] = m_new;
        if (tx == 0) alpha_s[r] = alpha;
      }
      __syncthreads();
      // O = alpha * O + P V
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float al = alpha_s[ty * 4 + i];
#pragma unroll
        for (int c = 0; c < DC; ++c) acc[i][c] *= al;
      }
      for (int kk = 0; kk < kT; ++kk) {
        float pv[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pv[i] = ss[(ty * 4 + i) * (kT + 1) + kk];
#pragma unroll
        for (int c = 0; c < DC; ++c) {
          const float vv = vs[kk * D + tx * DC + c];
#pragma unroll
          for (int i = 0; i < 4; ++i) acc[i][c] = fmaf(pv[i], vv, acc[i][c]);
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int row = q0 + ty * 4 + i;
    if (row >= p.Sq) continue;
    const float inv = 1.f / l_run[i];  // 0 -> inf -> NaN output, as the reference
    float* og = p.o + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(row) * p.o_ss;
#pragma unroll
    for (int c = 0; c < DC; ++c) og[tx * DC + c] = acc[i][c] * inv;
  }
}

int32_t bsa_fwd_simt(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                     const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                     int64_t col_capacity, int bm, int bn, const float* kv_bias,
                     int64_t bias_stride, float sm_scale, const int32_t* row_ranges,
                     cudaStream_t stream) {
  if (bm % kT != 0 || bn % kT != 0) return SAF_ERR_UNSUPPORTED;
  if (q->D != 64 && q->D != 128) return SAF_ERR_UNSUPPORTED;
  SimtParams p{};
  p.q = static_cast<const float*>(q->data);
  p.k = static_cast<const float*>(k->data);
  p.v = static_cast<const float*>(v->data);
  p.o = static_cast<float*>(o->data);
  p.H = static_cast<int>(q->H);
  p.Sq = static_cast<int>(q->S);
  p.Sk = static_cast<int>(k->S);
  p.q_sb = q->stride_b; p.q_sh = q->stride_h; p.q_ss = q->stride_s;
  p.k_sb = k->stride_b; p.k_sh = k->stride_h; p.k_ss = k->stride_s;
  p.v_sb = v->stride_b; p.v_sh = v->stride_h; p.v_ss = v->stride_s;
  p.o_sb = o->stride_b; p.o_sh = o->stride_h; p.o_ss = o->stride_s;
  p.bm = bm;
  p.bn = bn;
  p.nbq = static_cast<int>((q->S + bm - 1) / bm);
  p.nbk = static_cast<int>((k->S + bn - 1) / bn);
  p.col_capacity = col_capacity;
  p.row_ptr = row_ptr;
  p.col_idx = col_idx;
  p.kv_bias = kv_bias;
  p.bias_stride = bias_stride;
  p.scale = sm_scale;
  p.row_ranges = reinterpret_cast<const int4*>(row_ranges);
  p.status = device_status_ptr();
  if (p.status == nullptr) return SAF_ERR_CUDA;
  dim3 grid(static_cast<unsigned>((q->S + kT - 1) / kT), static_cast<unsigned>(q->B * q->H));
  if (q->D == 64) {
    const int smem = (3 * 64 * kT + kT * (kT + 1) + 2 * kT) * 4;
    SAF_CUDA_TRY(cudaFuncSetAttribute(bsa_fwd_simt_kernel<64>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    bsa_fwd_simt_kernel<64><<<grid, 256, smem, stream>>>(p);
  } else {
    const int smem = (3 * 128 * kT + kT * (kT + 1) + 2 * kT) * 4;
    SAF_CUDA_TRY(cudaFuncSetAttribute(bsa_fwd_simt_kernel<128>,
                                      cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    bsa_fwd_simt_kernel<128><<<grid, 256, smem, stream>>>(p);
  }
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

int32_t check_operand(const saf_tensor4* t, const saf_tensor4* ref) {
  int32_t rc = check_tensor4(t);
  if (rc != SAF_OK) return rc;
  if (t->dtype != ref->dtype) return SAF_ERR_DTYPE;
  if (t->B != ref->B || t->H != ref->H || t->D != ref->D) return SAF_ERR_SHAPE;
  return SAF_OK;
}

}  // namespace
}  // namespace saf

using namespace saf;

// Validation and dispatch shared by the attention entry points; `pool`
// (16-bit path only) asks for the pooled attention map.
int32_t bsa_fwd_entry(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                      const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                      int64_t col_capacity, int32_t block_m, int32_t block_n, const float* kv_bias,
                      int64_t kv_bias_stride_bh, float sm_scale, int32_t lead_rows,
                      const int32_t* row_ranges, const FrameMaskArgs* frames, const PoolArgs* pool,
                      void* stream) {
  int32_t rc = check_tensor4(q);
  if (rc != SAF_OK) return rc;
  if ((rc = check_operand(k, q)) != SAF_OK) return rc;
  if ((rc = check_operand(v, q)) != SAF_OK) return rc;
  if ((rc = check_operand(o, q)) != SAF_OK) return rc;
  if (k->S != v->S || o->S != q->S) return SAF_ERR_SHAPE;
  if (row_ptr == nullptr || col_idx == nullptr || col_capacity < 0) return SAF_ERR_ARG;
  if (block_m <= 0 || block_n <= 0) return SAF_ERR_ARG;
  if (kv_bias_stride_bh < 0) return SAF_ERR_STRIDE;
  if (lead_rows < 0) return SAF_ERR_ARG;
  if (q->S > 0x7fffffff || k->S > 0x7fffffff || q->B * q->H > 65535) return SAF_ERR_SHAPE;
  if (row_ranges != nullptr && (reinterpret_cast<uintptr_t>(row_ranges) & 15) != 0) return SAF_ERR_STRIDE;
  if (row_ranges != nullptr && kv_bias != nullptr) return SAF_ERR_UNSUPPORTED;
  if (frames != nullptr) {
    if (row_ranges != nullptr || kv_bias != nullptr || pool != nullptr) return SAF_ERR_UNSUPPORTED;
    if (frames->bits == nullptr) return SAF_ERR_ARG;
    if (frames->frames < 1 || frames->frames > 32 || frames->text_len < 0 || frames->frame_len < block_n ||
        q->S != k->S ||
        q->S != frames->text_len + static_cast<int64_t>(frames->frames) * frames->frame_len)
      return SAF_ERR_SHAPE;
    if (q->dtype == SAF_F32) return SAF_ERR_UNSUPPORTED;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (q->dtype == SAF_F32) {
    if (pool != nullptr) return SAF_ERR_UNSUPPORTED;
    DeviceScope dev_scope;
    if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
    return bsa_fwd_simt(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, kv_bias,
                        kv_bias_stride_bh, sm_scale, row_ranges, st);
  }
  // 16-bit path: tcgen05 kernel; tiles of 64 or 128, 16-byte aligned rows.
  if ((block_m != 64 && block_m != 128) || (block_n != 64 && block_n != 128))
    return SAF_ERR_UNSUPPORTED;
  const saf_tensor4* all[4] = {q, k, v, o};
  for (const saf_tensor4* t : all) {
    if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return SAF_ERR_STRIDE;
    if ((t->stride_s * 2) % 16 != 0 || (t->stride_h * 2) % 16 != 0 ||
        (t->stride_b * 2) % 16 != 0)
      return SAF_ERR_STRIDE;
  }
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
  // Leading mask rows -> leading 128-row query tiles scheduled first.
  const int64_t lead_tiles = (static_cast<int64_t>(lead_rows) * block_m + 127) / 128;
  return bsa_fwd_sm100(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, kv_bias,
                       kv_bias_stride_bh, sm_scale,
                       static_cast<int>(lead_tiles < 65535 ? lead_tiles : 65535), row_ranges,
                       frames, pool, st);
}

extern "C" int32_t saf_bsa_fwd_ranges(const saf_tensor4* q, const saf_tensor4* k,
                                      const saf_tensor4* v, const saf_tensor4* o,
                                      const int32_t* row_ptr, const int32_t* col_idx,
                                      int64_t col_capacity, int32_t block_m, int32_t block_n,
                                      const float* kv_bias, int64_t kv_bias_stride_bh,
                                      float sm_scale, int32_t lead_rows, const int32_t* row_ranges,
                                      void* stream) {
  return bsa_fwd_entry(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, kv_bias,
                       kv_bias_stride_bh, sm_scale, lead_rows, row_ranges, nullptr, nullptr, stream);
}

extern "C" int32_t saf_bsa_fwd_frames(const saf_tensor4* q, const saf_tensor4* k,
                                      const saf_tensor4* v, const saf_tensor4* o,
                                      const int32_t* row_ptr, const int32_t* col_idx,
                                      int64_t col_capacity, int32_t block_m, int32_t block_n,
                                      const uint32_t* frame_bits, int32_t text_len, int32_t frames,
                                      int32_t frame_len, float sm_scale, int32_t lead_rows,
                                      void* stream) {
  const FrameMaskArgs fm{frame_bits, text_len, frame_len, frames};
  return bsa_fwd_entry(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, nullptr, 0,
                       sm_scale, lead_rows, nullptr, &fm, nullptr, stream);
}

extern "C" int32_t saf_bsa_fwd(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                               const saf_tensor4* o, const int32_t* row_ptr,
                               const int32_t* col_idx, int64_t col_capacity, int32_t block_m,
                               int32_t block_n, const float* kv_bias, int64_t kv_bias_stride_bh,
                               float sm_scale, int32_t lead_rows, void* stream) {
  return saf_bsa_fwd_ranges(q, k, v, o, row_ptr, col_idx, col_capacity, block_m, block_n, kv_bias,
                            kv_bias_stride_bh, sm_scale, lead_rows, nullptr, stream);
}

extern "C" int32_t saf_bsa_fwd_keys(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                                    const saf_tensor4* o, const int32_t* key_list, int32_t key_len,
                                    const int32_t* key_batch, float sm_scale, void* stream) {
  int32_t rc;
  for (const saf_tensor4* t : {q, k, v, o})
    if ((rc = check_tensor4(t)) != SAF_OK) return rc;
  if (key_list == nullptr || key_batch == nullptr) return SAF_ERR_ARG;
  if (k->dtype != q->dtype || v->dtype != q->dtype || o->dtype != q->dtype) return SAF_ERR_DTYPE;
  if (q->dtype == SAF_F32) return SAF_ERR_UNSUPPORTED;
  if (v->B != k->B || v->H != k->H || v->S != k->S || k->H != q->H || k->D != q->D || v->D != q->D)
    return SAF_ERR_SHAPE;
  if (o->B != q->B || o->H != q->H || o->S != q->S || o->D != q->D) return SAF_ERR_SHAPE;
  if (key_len <= 0 || q->S > 0x7fffffff) return SAF_ERR_SHAPE;
  for (const saf_tensor4* t : {q, k, v, o})
    if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return SAF_ERR_STRIDE;
  if (o->stride_s % 8 != 0 || o->stride_h % 8 != 0 || o->stride_b % 8 != 0) return SAF_ERR_STRIDE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
  return bsa_fwd_sm100_keys(q, k, v, o, key_list, key_len, key_batch, sm_scale, static_cast<cudaStream_t>(stream));
}
