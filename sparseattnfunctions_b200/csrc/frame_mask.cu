// Frame-scope block masks (the reference's BlockSparseAttention.forward_backup
// path: generate_attention_mask_frame_scope, get_block_mask,
// special_attentions/utils/mask_related.py:194-245,397-404), built for the
// unpadded sequence [text | frames x frame_len].
//
// 1. frame_map_kernel: attention of the sampled tokens -- every text token
//    and, in each frame, the same n spatial positions -- to one another:
//    logits = scale * q_s . k_s (fp32 products of the stored values, fp32
//    sums) plus log(n / frame_len) on the text keys, softmax per query row
//    (fp64 sums of fp32 exponentials), and for each (query frame f1, key
//    frame f2) the video-video probability mass summed over the frame's
//    sampled queries.  A CTA takes one head, one query frame and a group of
//    its sampled rows: their logits against all sampled keys stay in shared
//    memory; each warp reduces its rows in a fixed order, the warps' sums are
//    added in warp order, and the groups' sums in group order, so the map is
//    the same on every run.
// 2. frame_select_kernel: per head, the frame map divided by n, sorted in
//    descending order (stable rank by counting), sequential fp64 cumulative
//    sum, and every entry ranked at or before the first position reaching
//    `threshold` of the total kept (the last position when none does): the
//    reference's rule (:222-243).  Output: the mask as bytes [F, F] and as
//    one word per query frame (bit f2 = key frame f2 visible).
// 3. frame_csr_kernel: per head, the 128- (or 64-) blocks of the sequence a
//    block of query rows may touch: every key block for a query block with a
//    text row, else the key blocks holding a text key or a key of a frame
//    that one of the query block's frames sees.  The attention kernel's
//    frame-mask mode then masks the exact keys inside each visited block.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cmath>
#include <cstdint>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kMapThreads = 256;
constexpr int kMapWarps = kMapThreads / 32;
constexpr int kMaxFrames = 32;

struct FrameMapParams {
  const void* q;
  const void* k;
  int32_t dtype;
  int64_t q_sb, q_sh, q_ss, k_sb, k_sh, k_ss;  // element strides
  int H, D;
  const int32_t* spatial;  // [n] positions inside a frame
  int n, T, F, FL;
  int nk;      // sampled keys: T + F * n
  int rows;    // sampled query rows per CTA
  int groups;  // CTAs per (head, query frame)
  float scale, comp;
  double* partial;  // [B*H, F, groups, F]
  unsigned int* status;
};

template <typename T>
__device__ __forceinline__ float to_f(T x);
template <>
__device__ __forceinline__ float to_f<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }
template <>
__device__ __forceinline__ float to_f<__half>(__half x) { return __half2float(x); }
template <>
__device__ __forceinline__ float to_f<float>(float x) { return x; }

// token index of sampled position j (keys: text first, then frame-major)
__device__ __forceinline__ int sampled_token(const FrameMapParams& p, int j) {
  if (j < p.T) return j;
  const int v = j - p.T, f = v / p.n;
  int s = __ldg(p.spatial + (v - f * p.n));
  if (s < 0 || s >= p.FL) {
    atomicOr(p.status, SAF_DEV_BADINDEX);
    s = 0;
  }
  return p.T + f * p.FL + s;
}

template <typename T, int D>
__global__ void __launch_bounds__(kMapThreads) frame_map_kernel(const FrameMapParams p) {
  extern __shared__ float fsm[];
  const int grp = blockIdx.x, f1 = blockIdx.y, g = blockIdx.z;
  const int b = g / p.H, h = g % p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r0 = grp * p.rows;
  const int nr = min(p.rows, p.n - r0);
  float* qs = fsm;                          // [rows][D]
  float* L = qs + p.rows * D;               // [rows][nk] logits, then exponentials
  double* wsum = reinterpret_cast<double*>(L + static_cast<int64_t>(p.rows) * p.nk + (p.rows * p.nk & 1));
  // wsum: [warps][F] this warp's sums over its rows
  const T* qb = static_cast<const T*>(p.q) + b * p.q_sb + h * p.q_sh;
  const T* kb = static_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;

  for (int i = threadIdx.x; i < nr * D; i += kMapThreads) {
    const int r = i / D, d = i - r * D;
    const int tok = sampled_token(p, p.T + f1 * p.n + r0 + r);
    qs[r * D + d] = to_f(qb[static_cast<int64_t>(tok) * p.q_ss + d]);
  }
  for (int i = threadIdx.x; i < kMapWarps * p.F; i += kMapThreads) wsum[i] = 0.0;
  __syncthreads();

  // logits: thread per sampled key, its row in registers
  for (int j = threadIdx.x; j < p.nk; j += kMapThreads) {
    const int tok = sampled_token(p, j);
    const T* kr = kb + static_cast<int64_t>(tok) * p.k_ss;
    float kv[D];
#pragma unroll
    for (int d = 0; d < D; ++d) kv[d] = to_f(kr[d]);
    const float add = j < p.T ? p.comp : 0.f;
    for (int r = 0; r < nr; ++r) {
      const float* qr = qs + r * D;
      float acc = 0.f;
#pragma unroll
      for (int d = 0; d < D; ++d) acc = fmaf(qr[d], kv[d], acc);
      L[static_cast<int64_t>(r) * p.nk + j] = acc * p.scale + add;
    }
  }
  __syncthreads();

  // per row: max, exponentials in place, fp64 total, per-frame video mass
  for (int r = warp; r < nr; r += kMapWarps) {
    float* lr = L + static_cast<int64_t>(r) * p.nk;
    float m = -INFINITY;
    for (int j = lane; j < p.nk; j += 32) m = fmaxf(m, lr[j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    double tot = 0.0;
    for (int j = lane; j < p.nk; j += 32) {
      const float e = expf(lr[j] - m);
      lr[j] = e;
      tot += static_cast<double>(e);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, off);
    __syncwarp();
    for (int f2 = 0; f2 < p.F; ++f2) {
      const float* seg = lr + p.T + f2 * p.n;
      double s = 0.0;
      for (int j = lane; j < p.n; j += 32) s += static_cast<double>(seg[j]);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (lane == 0) wsum[warp * p.F + f2] += s / tot;
    }
  }
  __syncthreads();
  for (int f2 = threadIdx.x; f2 < p.F; f2 += kMapThreads) {
    double s = 0.0;
    for (int w = 0; w < kMapWarps; ++w) s += wsum[w * p.F + f2];
    p.partial[((static_cast<int64_t>(g) * p.F + f1) * p.groups + grp) * p.F + f2] = s;
  }
}

struct FrameSelectParams {
  const double* partial;  // [BH, F, groups, F]
  int F, groups, n;
  double threshold;
  double* map_out;   // nullable [BH, F, F]
  uint8_t* mask_out; // nullable [BH, F, F]
  uint32_t* bits;    // [BH, F]
};

// One warp per head.
__global__ void __launch_bounds__(32) frame_select_kernel(const FrameSelectParams p) {
  __shared__ double val[kMaxFrames * kMaxFrames];
  __shared__ double sorted[kMaxFrames * kMaxFrames];
  __shared__ int16_t rank_of[kMaxFrames * kMaxFrames];
  __shared__ int kk_s;
  const int g = blockIdx.x, lane = threadIdx.x;
  const int N = p.F * p.F;
  for (int i = lane; i < N; i += 32) {
    const int f1 = i / p.F, f2 = i - f1 * p.F;
    const double* src = p.partial + (static_cast<int64_t>(g) * p.F + f1) * p.groups * p.F + f2;
    double s = 0.0;
    for (int gr = 0; gr < p.groups; ++gr) s += src[gr * p.F];
    val[i] = s / p.n;
    if (p.map_out != nullptr) p.map_out[static_cast<int64_t>(g) * N + i] = s / p.n;
  }
  __syncwarp();
  // stable descending rank: larger values first, ties to the lower index
  for (int i = lane; i < N; i += 32) {
    const double v = val[i];
    int r = 0;
    for (int j = 0; j < N; ++j) {
      const double u = val[j];
      r += (u > v) || (u == v && j < i);
    }
    rank_of[i] = static_cast<int16_t>(r);
    sorted[r] = v;
  }
  __syncwarp();
  if (lane == 0) {
    double tot = 0.0;
    for (int i = 0; i < N; ++i) tot += sorted[i];
    const double thr = p.threshold * tot;
    double cum = 0.0;
    int kk = N - 1;
    for (int i = 0; i < N; ++i) {
      cum += sorted[i];
      if (cum >= thr) {
        kk = i;
        break;
      }
    }
    kk_s = kk;
  }
  __syncwarp();
  const int kk = kk_s;
  for (int i = lane; i < N; i += 32)
    if (p.mask_out != nullptr) p.mask_out[static_cast<int64_t>(g) * N + i] = rank_of[i] <= kk ? 1 : 0;
  if (lane < p.F) {
    uint32_t w = 0;
    for (int f2 = 0; f2 < p.F; ++f2) w |= (rank_of[lane * p.F + f2] <= kk ? 1u : 0u) << f2;
    p.bits[static_cast<int64_t>(g) * p.F + lane] = w;
  }
}

struct FrameCsrParams {
  const uint32_t* bits;  // [BH, F]
  int T, F, FL;
  int S, bm, bn, nbq, nbk;
  int32_t* row_ptr;  // [BH, nbq + 1]
  int32_t* col_idx;  // head g's entries from g * nbq * nbk
};

__device__ __forceinline__ int frame_of(int tok, int T, int FL) { return tok < T ? -1 : (tok - T) / FL; }

// Frames of key block j as a bit mask; bit 31 of the result stands for text.
__device__ __forceinline__ uint32_t key_block_frames(const FrameCsrParams& p, int j) {
  const int c0 = j * p.bn, c1 = min(p.S, c0 + p.bn) - 1;
  const int a = frame_of(c0, p.T, p.FL), z = frame_of(c1, p.T, p.FL);
  uint32_t m = 0;
  for (int f = max(a, 0); f <= z; ++f) m |= 1u << f;
  if (a < 0) m |= 0x80000000u;
  return m;
}

// Key frames visible to some row of query block i; all (with the text bit)
// when the block holds a text row.
__device__ __forceinline__ uint32_t query_block_sees(const FrameCsrParams& p, const uint32_t* words, int i) {
  const int r0 = i * p.bm, r1 = min(p.S, r0 + p.bm) - 1;
  if (r0 < p.T) return 0xffffffffu;
  uint32_t m = 0x80000000u;  // text keys are always visible
  for (int f = frame_of(r0, p.T, p.FL); f <= frame_of(r1, p.T, p.FL); ++f) m |= words[f];
  return m;
}

constexpr int kCsrThreads = 256;

// One CTA per head: counts per query block, a sequential prefix, then the
// ascending column lists by warp ballots.
__global__ void __launch_bounds__(kCsrThreads) frame_csr_kernel(const FrameCsrParams p) {
  extern __shared__ int32_t csm[];
  int32_t* cnt = csm;  // [nbq + 1]
  __shared__ uint32_t words[kMaxFrames];
  const int g = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int warps = kCsrThreads / 32;
  if (threadIdx.x < p.F) words[threadIdx.x] = p.bits[static_cast<int64_t>(g) * p.F + threadIdx.x];
  __syncthreads();
  for (int i = warp; i < p.nbq; i += warps) {
    const uint32_t sees = query_block_sees(p, words, i);
    int c = 0;
    for (int j0 = 0; j0 < p.nbk; j0 += 32) {
      const int j = j0 + lane;
      const bool live = j < p.nbk && (key_block_frames(p, j) & sees) != 0;
      c += __popc(__ballot_sync(0xffffffffu, live));
    }
    if (lane == 0) cnt[i] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int32_t acc = 0;
    for (int i = 0; i < p.nbq; ++i) {
      const int32_t c = cnt[i];
      cnt[i] = acc;
      acc += c;
    }
    cnt[p.nbq] = acc;
  }
  __syncthreads();
  const int64_t base = static_cast<int64_t>(g) * p.nbq * p.nbk;
  int32_t* rp = p.row_ptr + static_cast<int64_t>(g) * (p.nbq + 1);
  for (int i = threadIdx.x; i <= p.nbq; i += kCsrThreads) rp[i] = static_cast<int32_t>(base + cnt[i]);
  for (int i = warp; i < p.nbq; i += warps) {
    const uint32_t sees = query_block_sees(p, words, i);
    int32_t at = cnt[i];
    for (int j0 = 0; j0 < p.nbk; j0 += 32) {
      const int j = j0 + lane;
      const bool live = j < p.nbk && (key_block_frames(p, j) & sees) != 0;
      const uint32_t bal = __ballot_sync(0xffffffffu, live);
      if (live) p.col_idx[base + at + __popc(bal & ((1u << lane) - 1u))] = j;
      at += __popc(bal);
    }
  }
}

int rows_per_cta(int nk, int D, int n) {
  // logits of `rows` rows + their q rows within ~160 KB of shared memory
  int r = (160 * 1024) / ((nk + D) * 4);
  r = r < 1 ? 1 : r;
  return r < n ? r : n;
}

size_t map_smem(int rows, int nk, int D, int F) {
  return static_cast<size_t>(rows) * D * 4 + (static_cast<size_t>(rows) * nk + 1) * 4 +
         static_cast<size_t>(kMapWarps) * F * 8 + 16;
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" size_t saf_frame_mask_workspace_bytes(int64_t BH, int32_t frames, int32_t n, int32_t text_len,
                                                 int32_t D) {
  if (BH <= 0 || frames <= 0 || n <= 0 || text_len < 0 || D <= 0) return 0;
  const int nk = text_len + frames * n;
  const int rows = rows_per_cta(nk, D, n);
  const int groups = (n + rows - 1) / rows;
  return static_cast<size_t>(BH) * frames * groups * frames * sizeof(double);
}

extern "C" int32_t saf_frame_mask(const saf_tensor4* q, const saf_tensor4* k, const int32_t* spatial,
                                  int32_t n, int32_t text_len, int32_t frames, int32_t frame_len,
                                  float sm_scale, double threshold, void* workspace,
                                  size_t workspace_bytes, double* map_out, uint8_t* mask_out,
                                  uint32_t* bits_out, void* stream) {
  int32_t rc = check_tensor4(q);
  if (rc != SAF_OK) return rc;
  if ((rc = check_tensor4(k)) != SAF_OK) return rc;
  if (k->dtype != q->dtype || k->B != q->B || k->H != q->H || k->D != q->D) return SAF_ERR_SHAPE;
  if (spatial == nullptr || bits_out == nullptr) return SAF_ERR_ARG;
  if (frames < 1 || frames > kMaxFrames || frame_len < 1 || text_len < 0 || n < 1 || n > frame_len)
    return SAF_ERR_SHAPE;
  if (q->D != 64 && q->D != 128) return SAF_ERR_UNSUPPORTED;
  const int64_t need_s = text_len + static_cast<int64_t>(frames) * frame_len;
  if (q->S < need_s || k->S < need_s) return SAF_ERR_SHAPE;
  if (!(threshold >= 0.0 && threshold <= 1.0)) return SAF_ERR_ARG;
  const int64_t BH = q->B * q->H;
  if (BH > 65535) return SAF_ERR_SHAPE;
  const size_t need = saf_frame_mask_workspace_bytes(BH, frames, n, text_len, static_cast<int32_t>(q->D));
  if (workspace == nullptr || workspace_bytes < need || (reinterpret_cast<uintptr_t>(workspace) & 7) != 0)
    return SAF_ERR_WORKSPACE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
  FrameMapParams p{};
  p.q = q->data;
  p.k = k->data;
  p.dtype = q->dtype;
  p.q_sb = q->stride_b, p.q_sh = q->stride_h, p.q_ss = q->stride_s;
  p.k_sb = k->stride_b, p.k_sh = k->stride_h, p.k_ss = k->stride_s;
  p.H = static_cast<int>(q->H);
  p.D = static_cast<int>(q->D);
  p.spatial = spatial;
  p.n = n, p.T = text_len, p.F = frames, p.FL = frame_len;
  p.nk = text_len + frames * n;
  p.rows = rows_per_cta(p.nk, p.D, n);
  p.groups = (n + p.rows - 1) / p.rows;
  p.scale = sm_scale;
  // log(n / frame_len) as a float32 value (the reference's float32 tensor)
  p.comp = logf(static_cast<float>(static_cast<double>(n) / frame_len));
  p.partial = static_cast<double*>(workspace);
  p.status = device_status_ptr();
  if (p.status == nullptr) return SAF_ERR_CUDA;
  const size_t smem = map_smem(p.rows, p.nk, p.D, frames);
  if (smem > 200 * 1024) return SAF_ERR_UNSUPPORTED;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(p.groups, frames, static_cast<unsigned>(BH));
#define SAF_FRAME_MAP(T_, D_)                                                                      \
  if (p.D == D_) {                                                                                 \
    SAF_CUDA_TRY(cudaFuncSetAttribute(frame_map_kernel<T_, D_>,                                    \
                                      cudaFuncAttributeMaxDynamicSharedMemorySize,                 \
                                      static_cast<int>(smem)));                                    \
    frame_map_kernel<T_, D_><<<grid, kMapThreads, smem, st>>>(p);                                  \
  }
  if (q->dtype == SAF_BF16) {
    SAF_FRAME_MAP(__nv_bfloat16, 64) SAF_FRAME_MAP(__nv_bfloat16, 128)
  } else if (q->dtype == SAF_F16) {
    SAF_FRAME_MAP(__half, 64) SAF_FRAME_MAP(__half, 128)
  } else {
    SAF_FRAME_MAP(float, 64) SAF_FRAME_MAP(float, 128)
  }
#undef SAF_FRAME_MAP
  SAF_CUDA_TRY(cudaGetLastError());
  FrameSelectParams s{p.partial, frames, p.groups, n, threshold, map_out, mask_out, bits_out};
  frame_select_kernel<<<static_cast<unsigned>(BH), 32, 0, st>>>(s);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

extern "C" int32_t saf_frame_csr(const uint32_t* bits, int64_t BH, int32_t text_len, int32_t frames,
                                 int32_t frame_len, int64_t S, int32_t block_m, int32_t block_n,
                                 int32_t* row_ptr, int32_t* col_idx, void* stream) {
  if (bits == nullptr || row_ptr == nullptr || col_idx == nullptr) return SAF_ERR_ARG;
  if (BH <= 0 || BH > 65535 || frames < 1 || frames > kMaxFrames - 1 || text_len < 0 || frame_len < 1)
    return SAF_ERR_SHAPE;
  if (S != text_len + static_cast<int64_t>(frames) * frame_len || S > 0x7fffffff) return SAF_ERR_SHAPE;
  if (block_m <= 0 || block_n <= 0 || frame_len < block_n) return SAF_ERR_SHAPE;
  const int64_t nbq = (S + block_m - 1) / block_m, nbk = (S + block_n - 1) / block_n;
  if (nbq > 16384 || BH * nbq * nbk >= (int64_t(1) << 31)) return SAF_ERR_SHAPE;
  DeviceScope dev_scope;
  int32_t rc = dev_scope.bind(bits);
  if (rc != SAF_OK) return rc;
  FrameCsrParams p{bits, text_len, frames, frame_len, static_cast<int>(S), block_m, block_n,
                   static_cast<int>(nbq), static_cast<int>(nbk), row_ptr, col_idx};
  const size_t smem = static_cast<size_t>(nbq + 1) * sizeof(int32_t);
  frame_csr_kernel<<<static_cast<unsigned>(BH), kCsrThreads, smem, static_cast<cudaStream_t>(stream)>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
