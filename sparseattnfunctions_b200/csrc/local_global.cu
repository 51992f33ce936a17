// Kernels of the local + global key selection of the reference's
// LocalGlobalAttention (special_attentions/LocalGlobalAttention.py:114-259),
// used with the probe kernel (probe_sm100.cu) and the attention kernel:
//
// 1. gather_rows_kernel: out[ob, h, s] = x[src / Sx, h, src % Sx] for
//    src = idx[ob, s] (a zero row for src < 0), 16-byte vectors.  Builds the
//    per-patch query rows and the per-(patch, batch) key / value lists
//    (transform_q, transform_kv_v1 :212-238), and puts the patch outputs back
//    in token order (transform_output :240-245) as a gather by the inverse
//    map.
// 2. masked_topn_kernel: per (patch, batch) row, the n keys of largest probe
//    mass outside the patch's local mask (the reference's masked_fill, sort
//    and slice, :58-62; ties to the lower key, as a stable descending sort),
//    listed in ascending key order: an 8-pass radix select on the
//    order-preserving bits of the fp64 mass, then two block scans place the
//    keys.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <cub/block/block_scan.cuh>

#include <cmath>
#include <cstdint>

#include "saf_common.cuh"

namespace saf {
namespace {

// ---------------------------------------------------------------- gather
struct GatherRowsParams {
  const uint4* x;
  uint4* out;
  int64_t x_sb, x_sh, x_ss;  // in 16-byte vectors
  int64_t o_sb, o_sh, o_ss;
  const int64_t* idx;  // [Bo, So]
  int64_t Sx, n_src;   // source rows per batch, total source rows (Bx * Sx)
  int H, So, vec;      // vectors per row
  int64_t rows;        // Bo * H * So
  unsigned int* status;
};

__global__ void __launch_bounds__(256) gather_rows_kernel(const GatherRowsParams p) {
  const int64_t n = p.rows * p.vec;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % p.vec);
    const int64_t row = i / p.vec;
    const int s = static_cast<int>(row % p.So);
    const int64_t bh = row / p.So;
    const int h = static_cast<int>(bh % p.H);
    const int64_t ob = bh / p.H;
    const int64_t src = p.idx[ob * p.So + s];
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (src >= p.n_src) {
      if (c == 0) atomicOr(p.status, SAF_DEV_BADINDEX);
    } else if (src >= 0) {
      const int64_t xb = src / p.Sx, xs = src % p.Sx;
      v = p.x[xb * p.x_sb + h * p.x_sh + xs * p.x_ss + c];
    }
    p.out[ob * p.o_sb + h * p.o_sh + static_cast<int64_t>(s) * p.o_ss + c] = v;
  }
}

// ---------------------------------------------------------------- top-n
constexpr int kTopThreads = 1024;

struct TopnParams {
  const double* mass;    // [B, Sk]
  const uint8_t* lmask;  // [P, Sk] keys of the row's local set (excluded)
  int B, Sk, n;
  int32_t* out;          // [P * B, n] ascending keys
};

// order-preserving 64-bit key of a non-negative double (larger -> larger);
// excluded keys map to 0, below every mass
__device__ __forceinline__ uint64_t mass_bits(double v) {
  return static_cast<uint64_t>(__double_as_longlong(v)) + 1ull;
}

__global__ void __launch_bounds__(kTopThreads) masked_topn_kernel(const TopnParams p) {
  using Scan = cub::BlockScan<int, kTopThreads>;
  __shared__ typename Scan::TempStorage scan_tmp;
  __shared__ int hist[256];
  __shared__ uint64_t s_prefix;
  __shared__ int s_need;
  const int r = blockIdx.x, pt = r / p.B, b = r % p.B, t = threadIdx.x;
  const double* mv = p.mass + static_cast<int64_t>(b) * p.Sk;
  const uint8_t* lm = p.lmask + static_cast<int64_t>(pt) * p.Sk;
  auto key_of = [&](int j) -> uint64_t {
    const double v = mv[j];
    return (lm[j] || !(v >= 0.0)) ? 0ull : mass_bits(v);
  };
  // radix select of the n-th largest key, 8 bits at a time from the top
  uint64_t prefix = 0ull, pmask = 0ull;
  int need = p.n;
  for (int shift = 56; shift >= 0; shift -= 8) {
    if (t < 256) hist[t] = 0;
    __syncthreads();
    for (int j = t; j < p.Sk; j += kTopThreads) {
      const uint64_t kv = key_of(j);
      if ((kv & pmask) == prefix) atomicAdd(&hist[(kv >> shift) & 255u], 1);
    }
    __syncthreads();
    if (t == 0) {
      int acc = 0, bin = 255;
      for (; bin > 0; --bin) {
        if (acc + hist[bin] >= need) break;
        acc += hist[bin];
      }
      s_prefix = prefix | (static_cast<uint64_t>(bin) << shift);
      s_need = need - acc;
    }
    __syncthreads();
    prefix = s_prefix;
    need = s_need;
    pmask |= 255ull << shift;
    __syncthreads();
  }
  // keys above the threshold, then `need` keys equal to it (lowest first);
  // each thread scans a contiguous run of keys so the output stays ascending
  const int per = (p.Sk + kTopThreads - 1) / kTopThreads;
  const int j0 = t * per, j1 = min(p.Sk, j0 + per);
  int gt = 0, eq = 0;
  for (int j = j0; j < j1; ++j) {
    const uint64_t kv = key_of(j);
    gt += kv > prefix;
    eq += kv == prefix && kv != 0ull;
  }
  int eq_before = 0, eq_total = 0;
  Scan(scan_tmp).ExclusiveSum(eq, eq_before, eq_total);
  __syncthreads();
  const int take_eq = max(0, min(eq, need - eq_before));
  int pos = 0, total = 0;
  Scan(scan_tmp).ExclusiveSum(gt + take_eq, pos, total);
  int32_t* o = p.out + static_cast<int64_t>(r) * p.n;
  int taken = 0;
  for (int j = j0; j < j1; ++j) {
    const uint64_t kv = key_of(j);
    if (kv > prefix || (kv == prefix && kv != 0ull && taken++ < take_eq)) {
      if (pos < p.n) o[pos] = j;
      ++pos;
    }
  }
  (void)total;
  (void)eq_total;
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" int32_t saf_gather_rows(const void* x, int32_t dtype, int64_t Bx, int64_t H, int64_t Sx, int64_t D,
                                   int64_t x_sb, int64_t x_sh, int64_t x_ss, void* out, int64_t Bo, int64_t So,
                                   int64_t o_sb, int64_t o_sh, int64_t o_ss, const int64_t* idx, void* stream) {
  if (x == nullptr || out == nullptr || idx == nullptr) return SAF_ERR_ARG;
  if (dtype != SAF_BF16 && dtype != SAF_F16 && dtype != SAF_F32) return SAF_ERR_DTYPE;
  if (Bx <= 0 || H <= 0 || Sx <= 0 || D <= 0 || Bo <= 0 || So <= 0) return SAF_ERR_SHAPE;
  const int64_t eb = elem_bytes(dtype);
  if ((D * eb) % 16 != 0 || (reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(out) & 15))
    return SAF_ERR_STRIDE;
  const int64_t v = 16 / eb;
  for (int64_t s : {x_sb, x_sh, x_ss, o_sb, o_sh, o_ss})
    if (s < 0 || s % v != 0) return SAF_ERR_STRIDE;
  if (H > 0x7fffffff || So > 0x7fffffff) return SAF_ERR_SHAPE;
  DeviceScope dev_scope;
  int32_t rc = dev_scope.bind(out);
  if (rc != SAF_OK) return rc;
  GatherRowsParams p{static_cast<const uint4*>(x), static_cast<uint4*>(out), x_sb / v, x_sh / v, x_ss / v,
                     o_sb / v, o_sh / v, o_ss / v, idx, Sx, Bx * Sx, static_cast<int>(H), static_cast<int>(So),
                     static_cast<int>(D * eb / 16), Bo * H * So, device_status_ptr()};
  if (p.status == nullptr) return SAF_ERR_CUDA;
  const int64_t work = p.rows * p.vec;
  const unsigned grid = static_cast<unsigned>(std::min<int64_t>((work + 255) / 256, 148 * 16));
  gather_rows_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

extern "C" int32_t saf_masked_topn(const double* mass, const uint8_t* local_mask, int64_t B, int64_t P,
                                   int64_t Sk, int32_t n, int32_t* out, void* stream) {
  if (mass == nullptr || local_mask == nullptr || out == nullptr) return SAF_ERR_ARG;
  if (B <= 0 || P <= 0 || Sk <= 0 || n <= 0 || n > Sk || P * B > 65535 || Sk > 0x7fffffff) return SAF_ERR_SHAPE;
  DeviceScope dev_scope;
  int32_t rc = dev_scope.bind(mass);
  if (rc != SAF_OK) return rc;
  TopnParams p{mass, local_mask, static_cast<int>(B), static_cast<int>(Sk), n, out};
  masked_topn_kernel<<<static_cast<unsigned>(P * B), kTopThreads, 0, static_cast<cudaStream_t>(stream)>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
