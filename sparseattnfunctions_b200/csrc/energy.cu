// Energy-threshold block selection (the adaptive-density mode of the
// reference's SparseGen_Plus processor).
//
// Per (head, row block) the estimated attention mass of every key block is
// sorted in descending order; the row keeps the smallest prefix whose fp64
// running sum reaches `threshold` of the row total (exactly as
// transfer_attn_to_mask(mode="energy"), SparseGen_Plus.py:52-78: the prefix
// ends before the first position where the running sum reaches the target,
// all columns if none does), clamped to [min_retain, max_retain]; then the
// first `text_blocks` rows and columns are forced live (:81-82).
//
// The mass comes either from the caller (`is_mass`, e.g. a sampled estimate)
// or from mean-pooled scores s (saf_pool_topk's fp64 scores): mass_j =
// n_j * exp(scale * s_j - max_j' scale * s_j'), n_j the key block's token
// count -- the softmax numerator of the pooled logits, weighted by block
// size.  The mass used is written out on request, so a checker can apply the
// reference rule to the very same values.
//
// One warp per row: values staged in shared memory, stable descending rank by
// counting (ties to the lower column), sequential fp64 prefix sum in sorted
// order by lane 0 (the reference's cumsum order), mask row written as bytes.
#include <cstdint>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kEnergyMaxN = 1024;
constexpr int kEnergyWarps = 4;

struct EnergyParams {
  const double* in;  // [rows, n]
  bool is_mass;
  int64_t rows;
  int nbq, n;        // row blocks per head, key blocks
  int block_n, Sk;
  double scale, threshold;
  int min_retain, max_retain, text_blocks;
  double* mass_out;  // nullable [rows, n]
  uint8_t* mask;     // [rows, n]
  // 0: energy rule; 1: adaptive top-k from init_k (transfer_attn_to_mask
  // mode "topk", SparseGen_Plus.py:28-50)
  int mode, init_k;
};

__global__ void __launch_bounds__(32 * kEnergyWarps) energy_select_kernel(const EnergyParams p) {
  extern __shared__ uint8_t esm[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kEnergyWarps + warp;
  if (row >= p.rows) return;
  const int n = p.n;
  double* val = reinterpret_cast<double*>(esm) + static_cast<int64_t>(warp) * n;
  int32_t* order = reinterpret_cast<int32_t*>(reinterpret_cast<double*>(esm) + kEnergyWarps * n) +
                   static_cast<int64_t>(warp) * n;
  uint8_t* keep = reinterpret_cast<uint8_t*>(reinterpret_cast<int32_t*>(
                      reinterpret_cast<double*>(esm) + kEnergyWarps * n) + kEnergyWarps * n) +
                  static_cast<int64_t>(warp) * n;
  const double* src = p.in + row * n;
  if (p.is_mass) {
    for (int j = lane; j < n; j += 32) val[j] = src[j];
  } else {
    double m = -INFINITY;
    for (int j = lane; j < n; j += 32) {
      const double l = p.scale * src[j];
      val[j] = l;
      m = fmax(m, l);
    }
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) m = fmax(m, __shfl_xor_sync(0xffffffffu, m, o));
    __syncwarp();
    for (int j = lane; j < n; j += 32) {
      const int cols = (j == n - 1) ? p.Sk - (n - 1) * p.block_n : p.block_n;
      val[j] = static_cast<double>(cols) * exp(val[j] - m);
    }
  }
  __syncwarp();
  if (p.mass_out)
    for (int j = lane; j < n; j += 32) p.mass_out[row * n + j] = val[j];
  // stable descending rank: larger values first, equal values by column
  for (int j = lane; j < n; j += 32) {
    const double v = val[j];
    int r = 0;
    for (int i = 0; i < n; ++i) {
      const double u = val[i];
      r += (u > v) || (u == v && i < j);
    }
    order[r] = j;
    keep[j] = 0;
  }
  __syncwarp();
  if (lane == 0) {
    // running sums in sorted order; total = the last running sum
    double cum = 0.0;
    double at_k = 0.0;  // running sum of the first init_k (topk mode)
    for (int r = 0; r < n; ++r) {
      cum = __dadd_rn(cum, val[order[r]]);
      if (r == p.init_k - 1) at_k = cum;
    }
    int k = n;
    if (p.mode == 1) {
      // grow the rows whose first init_k blocks hold under 60 % of the mass
      // to 3x, then cut every row under 90 % to 2/3 of its count
      k = p.init_k < n ? p.init_k : n;
      const bool grow = !(at_k >= __dmul_rn(0.6, cum)) && k < n;
      const bool cut = !(at_k >= __dmul_rn(0.9, cum)) && k < n;
      if (grow) k = 3 * k < n ? 3 * k : n;
      if (cut) k = (k / 3) * 2 < n ? (k / 3) * 2 : n;
    } else {
      const double target = __dmul_rn(p.threshold, cum);
      double run = 0.0;
      for (int r = 0; r < n; ++r) {
        run = __dadd_rn(run, val[order[r]]);
        if (run >= target) {
          k = r;
          break;
        }
      }
      k = k < p.min_retain ? p.min_retain : k;
      k = k > p.max_retain ? p.max_retain : k;
      k = k > n ? n : k;
    }
    for (int r = 0; r < k; ++r) keep[order[r]] = 1;
  }
  __syncwarp();
  const bool text_row = static_cast<int>(row % p.nbq) < p.text_blocks;
  uint8_t* mrow = p.mask + row * n;
  for (int j = lane; j < n; j += 32) mrow[j] = (text_row || j < p.text_blocks || keep[j]) ? 1 : 0;
}

}  // namespace
}  // namespace saf

using namespace saf;

namespace {
int32_t select_entry(const double* in, int32_t is_mass, int64_t BH, int32_t nbq, int32_t nbk,
                     int32_t block_n, int64_t Sk, double scale, double threshold, int32_t min_retain,
                     int32_t max_retain, int32_t text_blocks, double* mass_out, uint8_t* mask, int mode,
                     int32_t init_k, void* stream) {
  if (in == nullptr || mask == nullptr) return SAF_ERR_ARG;
  if (BH <= 0 || nbq <= 0 || nbk <= 0 || nbk > kEnergyMaxN) return SAF_ERR_SHAPE;
  if (!is_mass && (block_n <= 0 || Sk <= static_cast<int64_t>(nbk - 1) * block_n ||
                   Sk > static_cast<int64_t>(nbk) * block_n))
    return SAF_ERR_SHAPE;
  if (min_retain < 0 || max_retain < 0 || text_blocks < 0) return SAF_ERR_ARG;
  if (mode == 1 && (init_k < 1 || init_k > nbk)) return SAF_ERR_ARG;
  int32_t rc;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(in)) != SAF_OK) return rc;
  EnergyParams p{in, is_mass != 0, BH * nbq, nbq, nbk, block_n, static_cast<int>(Sk), scale, threshold,
                 min_retain, max_retain, text_blocks, mass_out, mask, mode, mode == 1 ? init_k : 0};
  const int64_t rows = BH * nbq;
  const size_t smem = static_cast<size_t>(kEnergyWarps) * nbk * (8 + 4 + 1);
  if (smem > 48 * 1024)
    SAF_CUDA_TRY(cudaFuncSetAttribute(energy_select_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)));
  energy_select_kernel<<<static_cast<unsigned>((rows + kEnergyWarps - 1) / kEnergyWarps), 32 * kEnergyWarps,
                         smem, static_cast<cudaStream_t>(stream)>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
}  // namespace

extern "C" int32_t saf_energy_select(const double* in, int32_t is_mass, int64_t BH, int32_t nbq,
                                     int32_t nbk, int32_t block_n, int64_t Sk, double scale,
                                     double threshold, int32_t min_retain, int32_t max_retain,
                                     int32_t text_blocks, double* mass_out, uint8_t* mask,
                                     void* stream) {
  return select_entry(in, is_mass, BH, nbq, nbk, block_n, Sk, scale, threshold, min_retain, max_retain,
                      text_blocks, mass_out, mask, 0, 0, stream);
}

extern "C" int32_t saf_topk_adaptive_select(const double* in, int32_t is_mass, int64_t BH, int32_t nbq,
                                            int32_t nbk, int32_t block_n, int64_t Sk, double scale,
                                            int32_t init_k, int32_t text_blocks, double* mass_out,
                                            uint8_t* mask, void* stream) {
  return select_entry(in, is_mass, BH, nbq, nbk, block_n, Sk, scale, 0.0, 0, 0, text_blocks, mass_out,
                      mask, 1, init_k, stream);
}
