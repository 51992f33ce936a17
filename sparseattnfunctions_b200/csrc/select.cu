// select.cu -- block selection: mean-pool q and k per block, score the pooled
// blocks, keep the top-k columns per row block, force text rows / columns,
// and emit a segmented CSR.  Also the dense-mask -> CSR conversion.
//
// Numerics contract (shared with the CPU oracle, oracle/selection.py):
//   * block means: fp64 sum of the block's rows (exact for realistic data:
//     bf16 / f16 values summed in fp64 lose nothing unless the block spans
//     more than ~2^40 in magnitude), divided by the valid row count
//     (IEEE division);
//   * score[i][j] = sum_d q_mean[i][d] * k_mean[j][d] in fp64, d ascending,
//     every product and every sum rounded separately (no FMA contraction);
//   * top-k order: higher score first, equal scores -> lower column first,
//     NaN above every number (torch.topk's rule; NaNs tie among themselves).
// With these rules the GPU and the oracle select bit-identical blocks.
//
// Reference counterparts: calc_attn_block_sum_efficient
// (special_attentions/utils/mask_related.py:40-81) pools a random 8-of-64
// token sample per block; the deterministic mean-pool replaces it.
// get_sparse_attn_mask_from_topk (utils/block_sparse_attn_kernel.py:31-39)
// is the top-k rule; transfer_attn_to_mask (SparseGen_Plus.py:81-82) and
// get_block_mask (utils/mask_related.py:402-403) force the text blocks.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <mutex>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kPoolThreads = 256;
constexpr int kMaxM = 16;  // column slots per lane: nbk <= 512
constexpr int kDChunk = 32;

__device__ __forceinline__ double to_f64(__nv_bfloat16 x) {
  return static_cast<double>(__bfloat162float(x));
}
__device__ __forceinline__ double to_f64(__half x) { return static_cast<double>(__half2float(x)); }
__device__ __forceinline__ double to_f64(float x) { return static_cast<double>(x); }

struct PoolOperand {
  const void* x;
  int S;
  int64_t sb, sh, ss;
  int block, nb;
  double* out;  // [B*H, nb, D]
};

// One warp per (head, block): lanes hold 16-byte column chunks of 32 / lpr
// rows at a time (lpr = lanes per row, a power of two), accumulate in fp64,
// and combine the row groups with xor shuffles -- no shared memory and no
// block barrier, so the many small blocks cost no per-CTA synchronisation.
// grid (ceil(B*H*max nb / 8), 1, 2): z = 0 pools q, z = 1 pools k.
template <typename T>
__global__ void __launch_bounds__(256, 2) pool_mean_warp_kernel(PoolOperand q_op, PoolOperand k_op, int H,
                                                             int D, int BH, int lpr_log2) {
  constexpr int VEC = 16 / sizeof(T);
  constexpr int U = 8;  // row loads in flight per lane (6 at three CTAs per SM: 1 us slower at 8 heads)
  const PoolOperand& op = blockIdx.z == 0 ? q_op : k_op;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t wid = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  if (wid >= static_cast<int64_t>(BH) * op.nb) return;
  const int g = static_cast<int>(wid / op.nb), blk = static_cast<int>(wid % op.nb);
  const int b = g / H, h = g % H;
  const int lpr = 1 << lpr_log2, rpi = 32 >> lpr_log2;
  const int c = lane & (lpr - 1), ro = lane >> lpr_log2;
  const int r0 = blk * op.block;
  const int nrows = min(op.block, op.S - r0);
  const T* base = static_cast<const T*>(op.x) + static_cast<int64_t>(b) * op.sb +
                  static_cast<int64_t>(h) * op.sh + static_cast<int64_t>(r0) * op.ss + c * VEC;
  double acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc[e] = 0.0;
  for (int r = ro; r < nrows; r += rpi * U) {
    uint4 v[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int rr = r + u * rpi;
      v[u] = rr < nrows ? __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(rr) * op.ss))
                        : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const T* pv = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] += to_f64(pv[e]);
    }
  }
  for (int m = lpr; m < 32; m <<= 1)
#pragma unroll
    for (int e = 0; e < VEC; ++e) acc[e] += __shfl_xor_sync(0xffffffffu, acc[e], m);
  if (ro == 0) {
    double* o = op.out + (static_cast<int64_t>(g) * op.nb + blk) * D + c * VEC;
#pragma unroll
    for (int e = 0; e < VEC; ++e) o[e] = acc[e] / static_cast<double>(nrows);
  }
}

// grid (max nb, B*H, 2): z = 0 pools q, z = 1 pools k.  Mean over the rows of
// one block in fp64.  Each thread owns one 16-byte column chunk and issues all
// of its row loads before accumulating, so a CTA keeps the whole block in
// flight.
template <typename T, int kMaxRowsPerThread>
__global__ void __launch_bounds__(kPoolThreads) pool_mean_kernel(PoolOperand q_op,
                                                                 PoolOperand k_op, int H, int D) {
  constexpr int VEC = 16 / sizeof(T);
  extern __shared__ double part[];  // [groups][D]
  const PoolOperand& op = blockIdx.z == 0 ? q_op : k_op;
  const int blk = blockIdx.x, g = blockIdx.y;
  if (blk >= op.nb) return;
  const int b = g / H, h = g % H;
  const int r0 = blk * op.block;
  const int nrows = min(op.block, op.S - r0);
  const int vpr = D / VEC;                // vectors per row
  const int groups = kPoolThreads / vpr;  // rows processed in parallel
  const int tid = threadIdx.x;
  const int vc = tid % vpr, rg = tid / vpr;
  const T* base = static_cast<const T*>(op.x) + static_cast<int64_t>(b) * op.sb +
                  static_cast<int64_t>(h) * op.sh + static_cast<int64_t>(r0) * op.ss + vc * VEC;
  double acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; ++e) acc[e] = 0.0;
  // Threads past `groups` rows (D / VEC not dividing the block size) idle.
  for (int r = rg; rg < groups && r < nrows; r += groups * kMaxRowsPerThread) {
    uint4 v[kMaxRowsPerThread];
#pragma unroll
    for (int u = 0; u < kMaxRowsPerThread; ++u) {
      const int rr = r + u * groups;
      v[u] = rr < nrows ? __ldg(reinterpret_cast<const uint4*>(base + static_cast<int64_t>(rr) * op.ss))
                        : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kMaxRowsPerThread; ++u) {
      const T* pv = reinterpret_cast<const T*>(&v[u]);
#pragma unroll
      for (int e = 0; e < VEC; ++e) acc[e] += to_f64(pv[e]);
    }
  }
  if (rg < groups) {
#pragma unroll
    for (int e = 0; e < VEC; ++e) part[rg * D + vc * VEC + e] = acc[e];
  }
  __syncthreads();
  for (int d = tid; d < D; d += kPoolThreads) {
    double s = 0.0;
    for (int k = 0; k < groups; ++k) s += part[k * D + d];
    op.out[(static_cast<int64_t>(g) * op.nb + blk) * D + d] = s / static_cast<double>(nrows);
  }
}

struct SelectArgs {
  int nbq, nbk, D;
  int dc;  // dimensions staged per pass (divides D)
  int topk, text_q, text_k, force_diag, forced_inside;
  const double* qbar;  // [BH, nbq, D]
  const double* kbar;  // [BH, nbk, D]
  int32_t* padded;     // [BH, nbq, nbk]
  int32_t* counts;     // [BH, nbq]
  uint8_t* mask_out;   // nullable [BH, nbq, nbk]
  double* score_out;   // nullable [BH, nbq, nbk]
};

// 16-byte asynchronous global -> shared copy, cached in L2 only.
__device__ __forceinline__ void cp_async16(double* dst, const double* src) {
  const uint32_t d = static_cast<uint32_t>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(d), "l"(src) : "memory");
}

// Order-preserving 64-bit key of a score: larger score <-> larger key, -0.0
// keyed as +0.0 (the two compare equal), NaN keyed above +inf (torch.topk,
// which the reference selects with, ranks NaN highest; all NaNs tie, so the
// lower column goes first), 0 reserved for columns outside the top-k pool.
// Every candidate keys to at least 0x000FFFFFFFFFFFFF, so its high word is
// never 0.
__device__ __forceinline__ unsigned long long score_key(double s, bool candidate) {
  const double c = __dadd_rn(s, 0.0);  // -0.0 + 0.0 == +0.0; any other value unchanged
  const unsigned long long b = static_cast<unsigned long long>(__double_as_longlong(c));
  if (!candidate) return 0ull;
  if (c != c) return ~0ull;
  return (b >> 63) ? ~b : (b | 0x8000000000000000ull);
}

// grid (B*H, ceil(nbq / (8 RPW))), 256 threads; each warp owns RPW
// consecutive row blocks.  The head's key means and the CTA's query means
// are staged in shared memory dc dimensions at a time (dc = D whenever both
// fit in ~100 KB, two CTAs per SM) by 16-byte cp.async copies, all in flight
// at once, into rows of dc + 2 doubles: a lane's 16-byte read of (d, d + 1)
// then falls in a different bank group for each of 8 consecutive rows, so a
// warp's read of 32 columns is conflict-free.  Every lane owns columns
// lane + 32m (m < M) and accumulates their fp64 scores with d ascending
// (separate multiply and add, no contraction); one shared-memory read of a
// key pair serves RPW rows.  Lanes past the last column read the last
// column's row (their scores are never candidates).
//
// The top-k is k rounds of a warp arg-max over order-preserving 64-bit keys
// of the scores, the RPW rows of a warp advancing together: redux.sync max of
// the lanes' best high words, and a ballot of the lanes holding it; when one
// lane holds it, that lane's best is the winner, otherwise the low words and
// then the lowest column among equal keys decide.  Only the lane that owned
// the winner rescans its columns.
template <int M, int RPW>
__global__ void __launch_bounds__(256) score_topk_kernel(const SelectArgs a) {
  constexpr int kRowsPerCta = 8 * RPW;
  extern __shared__ __align__(16) double ks[];  // [nbk][dc + 2] then [kRowsPerCta][dc + 2]
  const int dc = a.dc, ld = a.dc + 2, half = a.dc >> 1;
  double* qs = ks + a.nbk * ld;
  const int g = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int cta_row0 = blockIdx.y * kRowsPerCta;
  const int row0 = cta_row0 + warp * RPW;
  const int qrows = min(kRowsPerCta, a.nbq - cta_row0);

  double sc[RPW][M];
#pragma unroll
  for (int i = 0; i < RPW; ++i)
#pragma unroll
    for (int m = 0; m < M; ++m) sc[i][m] = 0.0;
  int koff[M];
#pragma unroll
  for (int m = 0; m < M; ++m) koff[m] = min(lane + 32 * m, a.nbk - 1) * ld;

  const double* kb = a.kbar + static_cast<int64_t>(g) * a.nbk * a.D;
  const double* qb = a.qbar + (static_cast<int64_t>(g) * a.nbq + cta_row0) * a.D;
  const double* qr = qs + warp * RPW * ld;
  for (int d0 = 0; d0 < a.D; d0 += dc) {
    if (d0 > 0) __syncthreads();  // every warp is done with the previous pass
    for (int j = warp; j < a.nbk; j += 8)
      for (int c = lane; c < half; c += 32)
        cp_async16(ks + j * ld + 2 * c, kb + static_cast<int64_t>(j) * a.D + d0 + 2 * c);
    for (int r = warp; r < qrows; r += 8)
      for (int c = lane; c < half; c += 32)
        cp_async16(qs + r * ld + 2 * c, qb + static_cast<int64_t>(r) * a.D + d0 + 2 * c);
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
    __syncthreads();
#pragma unroll 2
    for (int d = 0; d < dc; d += 2) {
      double2 qv[RPW];
#pragma unroll
      for (int i = 0; i < RPW; ++i) qv[i] = *reinterpret_cast<const double2*>(qr + i * ld + d);
#pragma unroll
      for (int m = 0; m < M; ++m) {
        const double2 kv = *reinterpret_cast<const double2*>(ks + koff[m] + d);
#pragma unroll
        for (int i = 0; i < RPW; ++i) {
          sc[i][m] = __dadd_rn(sc[i][m], __dmul_rn(qv[i].x, kv.x));
          sc[i][m] = __dadd_rn(sc[i][m], __dmul_rn(qv[i].y, kv.y));
        }
      }
    }
  }

  // Per row: forced / candidate columns, the keys, and the lane's best key.
  uint32_t forced[RPW], sel[RPW];
  int krem[RPW];
  unsigned long long key[RPW][M], bk[RPW];
  int bm[RPW];
#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int row = row0 + i;
    const bool live_row = row < a.nbq;
    const bool text_row = row < a.text_q;
    uint32_t eligible = 0;
    forced[i] = 0;
    sel[i] = 0;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const int j = lane + 32 * m;
      if (j < a.nbk) {
        const bool f = text_row || j < a.text_k || (a.force_diag && j == row);
        if (f) forced[i] |= 1u << m;
        if (!(f && a.forced_inside)) eligible |= 1u << m;
      }
    }
    int nforced = 0;
#pragma unroll
    for (int m = 0; m < M; ++m) nforced += __popc(__ballot_sync(0xffffffffu, (forced[i] >> m) & 1u));
    krem[i] = a.forced_inside ? a.topk - nforced : a.topk;
    if (text_row || !live_row) krem[i] = 0;
    if (live_row && a.score_out) {
      const int64_t rbase = (static_cast<int64_t>(g) * a.nbq + row) * a.nbk;
#pragma unroll
      for (int m = 0; m < M; ++m)
        if (lane + 32 * m < a.nbk) a.score_out[rbase + lane + 32 * m] = sc[i][m];
    }
    bk[i] = 0ull;
    bm[i] = 0;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      key[i][m] = score_key(sc[i][m], (eligible >> m) & 1u);
      if (key[i][m] > bk[i]) {
        bk[i] = key[i][m];
        bm[i] = m;
      }
    }
  }
  int kmax = 0;
#pragma unroll
  for (int i = 0; i < RPW; ++i) kmax = max(kmax, krem[i]);
  for (int round = 0; round < kmax; ++round) {
    uint32_t hi[RPW], holders[RPW];
#pragma unroll
    for (int i = 0; i < RPW; ++i) hi[i] = __reduce_max_sync(0xffffffffu, static_cast<uint32_t>(bk[i] >> 32));
#pragma unroll
    for (int i = 0; i < RPW; ++i)
      holders[i] = __ballot_sync(0xffffffffu, static_cast<uint32_t>(bk[i] >> 32) == hi[i]);
#pragma unroll
    for (int i = 0; i < RPW; ++i) {
      if (round >= krem[i] || hi[i] == 0u) continue;  // row done, or no candidate left (uniform)
      bool win;
      if (__popc(holders[i]) == 1) {
        win = lane == __ffs(holders[i]) - 1;
      } else {
        const bool top = (holders[i] >> lane) & 1u;
        const uint32_t lo = __reduce_max_sync(0xffffffffu, top ? static_cast<uint32_t>(bk[i]) : 0u);
        const bool hold = top && static_cast<uint32_t>(bk[i]) == lo;
        const uint32_t col =
            __reduce_min_sync(0xffffffffu, hold ? static_cast<uint32_t>(lane + 32 * bm[i]) : 0xffffffffu);
        win = (col & 31u) == static_cast<uint32_t>(lane);
      }
      if (win) {
        sel[i] |= 1u << bm[i];
        bk[i] = 0ull;
        bm[i] = 0;
#pragma unroll
        for (int m = 0; m < M; ++m)
          if (!((sel[i] >> m) & 1u) && key[i][m] > bk[i]) {
            bk[i] = key[i][m];
            bm[i] = m;
          }
      }
    }
  }

#pragma unroll
  for (int i = 0; i < RPW; ++i) {
    const int row = row0 + i;
    if (row >= a.nbq) break;
    const int64_t rbase = (static_cast<int64_t>(g) * a.nbq + row) * a.nbk;
    const uint32_t s = sel[i] | forced[i];
    int base = 0;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const uint32_t bal = __ballot_sync(0xffffffffu, (s >> m) & 1u);
      if ((s >> m) & 1u) {
        const int pos = base + __popc(bal & ((1u << lane) - 1u));
        a.padded[rbase + pos] = lane + 32 * m;
      }
      base += __popc(bal);
      if (a.mask_out && lane + 32 * m < a.nbk) a.mask_out[rbase + lane + 32 * m] = (s >> m) & 1u;
    }
    if (lane == 0) a.counts[static_cast<int64_t>(g) * a.nbq + row] = base;
  }
}

// grid (B*H, ceil(nbq / 8)), 256 threads.  Every CTA redoes the (small)
// exclusive scan of its head's row counts, then one warp per row copies that
// row's columns into its CSR slot.  CTA y == 0 also writes the head's row_ptr.
__global__ void __launch_bounds__(256) csr_compact_kernel(int nbq, int nbk,
                                                          const int32_t* __restrict__ counts,
                                                          const int32_t* __restrict__ padded,
                                                          int32_t* __restrict__ row_ptr,
                                                          int32_t* __restrict__ col_idx) {
  __shared__ int32_t pref[1025];
  __shared__ int32_t warp_tot[8];
  const int g = blockIdx.x;
  const int64_t seg = static_cast<int64_t>(g) * nbq * nbk;
  const int32_t* cnt = counts + static_cast<int64_t>(g) * nbq;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  int local[4], tot = 0;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int r = tid * 4 + e;
    local[e] = r < nbq ? cnt[r] : 0;
    tot += local[e];
  }
  int incl = tot;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  int wbase = 0;
  for (int w = 0; w < warp; ++w) wbase += warp_tot[w];
  int run = wbase + incl - tot;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int r = tid * 4 + e;
    if (r < nbq) pref[r] = run;
    run += local[e];
  }
  if (tid == 255) pref[nbq] = run;  // the last thread holds the grand total
  __syncthreads();
  if (blockIdx.y == 0) {
    int32_t* rp = row_ptr + static_cast<int64_t>(g) * (nbq + 1);
    for (int r = tid; r <= nbq; r += 256) rp[r] = static_cast<int32_t>(seg + pref[r]);
  }
  const int r = blockIdx.y * 8 + warp;
  if (r < nbq) {
    const int n = pref[r + 1] - pref[r];
    const int32_t* src = padded + seg + static_cast<int64_t>(r) * nbk;
    int32_t* dst = col_idx + seg + pref[r];
    for (int c = lane; c < n; c += 32) dst[c] = src[c];
  }
}

// grid (B*H), 512 threads: dense uint8 mask -> segmented CSR for one head.
// Pass 1 counts every row, a block scan turns counts into offsets, pass 2
// writes the columns (ascending) at their offsets.
__global__ void __launch_bounds__(512) mask_to_csr_kernel(const uint8_t* __restrict__ mask,
                                                          int nbq, int nbk, int64_t s_bh,
                                                          int64_t s_row, int32_t* __restrict__ row_ptr,
                                                          int32_t* __restrict__ col_idx) {
  extern __shared__ int32_t cnt_s[];  // [nbq + 1]
  const int g = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nwarps = blockDim.x >> 5;
  const uint8_t* mg = mask + static_cast<int64_t>(g) * s_bh;
  for (int r = warp; r < nbq; r += nwarps) {
    int c = 0;
    for (int j0 = 0; j0 < nbk; j0 += 32) {
      const int j = j0 + lane;
      c += __popc(__ballot_sync(0xffffffffu, j < nbk && mg[static_cast<int64_t>(r) * s_row + j]));
    }
    if (lane == 0) cnt_s[r] = c;
  }
  __syncthreads();
  if (threadIdx.x == 0) {  // nbq is small (<= a few hundred): serial scan
    int run = 0;
    for (int r = 0; r < nbq; ++r) {
      const int c = cnt_s[r];
      cnt_s[r] = run;
      run += c;
    }
    cnt_s[nbq] = run;
  }
  __syncthreads();
  const int64_t seg = static_cast<int64_t>(g) * nbq * nbk;
  int32_t* rp = row_ptr + static_cast<int64_t>(g) * (nbq + 1);
  for (int r = threadIdx.x; r <= nbq; r += blockDim.x) rp[r] = static_cast<int32_t>(seg + cnt_s[r]);
  for (int r = warp; r < nbq; r += nwarps) {
    int base = cnt_s[r];
    for (int j0 = 0; j0 < nbk; j0 += 32) {
      const int j = j0 + lane;
      const bool on = j < nbk && mg[static_cast<int64_t>(r) * s_row + j];
      const uint32_t bal = __ballot_sync(0xffffffffu, on);
      if (on) col_idx[seg + base + __popc(bal & ((1u << lane) - 1u))] = j;
      base += __popc(bal);
    }
  }
}

struct SelectLayout {
  size_t off_qbar, off_kbar, off_padded, off_counts, total;
};

SelectLayout select_layout(int64_t BH, int nbq, int nbk, int D) {
  auto up = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  SelectLayout l{};
  l.off_qbar = 0;
  l.off_kbar = up(l.off_qbar + static_cast<size_t>(BH) * nbq * D * sizeof(double));
  l.off_padded = up(l.off_kbar + static_cast<size_t>(BH) * nbk * D * sizeof(double));
  l.off_counts = up(l.off_padded + static_cast<size_t>(BH) * nbq * nbk * sizeof(int32_t));
  l.total = up(l.off_counts + static_cast<size_t>(BH) * nbq * sizeof(int32_t));
  return l;
}

template <typename T>
int32_t launch_pool_t(const saf_tensor4* q, const saf_tensor4* k, int bm, int bn, int nbq, int nbk,
                      double* qbar, double* kbar, cudaStream_t st) {
  constexpr int VEC = 16 / sizeof(T);
  const int D = static_cast<int>(q->D);
  const int vpr = D / VEC;
  const int groups = kPoolThreads / vpr;
  const size_t smem = static_cast<size_t>(groups) * D * sizeof(double);
  PoolOperand qo{q->data, static_cast<int>(q->S), q->stride_b, q->stride_h, q->stride_s, bm, nbq, qbar};
  PoolOperand ko{k->data, static_cast<int>(k->S), k->stride_b, k->stride_h, k->stride_s, bn, nbk, kbar};
  const int BH = static_cast<int>(q->B * q->H);
  if (vpr <= 32 && (vpr & (vpr - 1)) == 0) {  // lanes per row: a power of two
    int lg = 0;
    while ((1 << lg) < vpr) ++lg;
    const int64_t pairs = static_cast<int64_t>(BH) * (nbq > nbk ? nbq : nbk);
    dim3 wgrid(static_cast<unsigned>((pairs + 7) / 8), 1, 2);
    pool_mean_warp_kernel<T><<<wgrid, 256, 0, st>>>(qo, ko, static_cast<int>(q->H), D, BH, lg);
    return SAF_OK;
  }
  dim3 grid(nbq > nbk ? nbq : nbk, static_cast<unsigned>(q->B * q->H), 2);
  // rows per thread per pass: the whole block in one pass when it fits in 8
  const int bmax = bm > bn ? bm : bn;
  if ((bmax + groups - 1) / groups <= 4) {
    pool_mean_kernel<T, 4><<<grid, kPoolThreads, smem, st>>>(qo, ko, static_cast<int>(q->H), D);
  } else {
    pool_mean_kernel<T, 8><<<grid, kPoolThreads, smem, st>>>(qo, ko, static_cast<int>(q->H), D);
  }
  return SAF_OK;
}

int32_t check_pool_operand(const saf_tensor4* t) {
  int32_t rc = check_tensor4(t);
  if (rc != SAF_OK) return rc;
  const int eb = elem_bytes(t->dtype);
  const int vec = 16 / eb;
  if (t->D % vec != 0 || t->D > 256 || (kPoolThreads / (t->D / vec)) < 1) return SAF_ERR_SHAPE;
  if ((reinterpret_cast<uintptr_t>(t->data) & 15) != 0) return SAF_ERR_STRIDE;
  if ((t->stride_s * eb) % 16 != 0 || (t->stride_h * eb) % 16 != 0 || (t->stride_b * eb) % 16 != 0)
    return SAF_ERR_STRIDE;
  return SAF_OK;
}

int32_t pool_dispatch(const saf_tensor4* q, const saf_tensor4* k, int bm, int bn, int nbq, int nbk,
                      double* qbar, double* kbar, cudaStream_t st) {
  switch (q->dtype) {
    case SAF_BF16: return launch_pool_t<__nv_bfloat16>(q, k, bm, bn, nbq, nbk, qbar, kbar, st);
    case SAF_F16: return launch_pool_t<__half>(q, k, bm, bn, nbq, nbk, qbar, kbar, st);
    case SAF_F32: return launch_pool_t<float>(q, k, bm, bn, nbq, nbk, qbar, kbar, st);
    default: return SAF_ERR_DTYPE;
  }
}

template <int M, int RPW>
int32_t launch_score_rpw(SelectArgs a, int64_t BH, cudaStream_t st) {
  constexpr int kRowsPerCta = 8 * RPW;
  constexpr size_t kSmemTarget = 100 * 1024;  // two CTAs per SM
  auto smem_of = [&](int dc) {
    return (static_cast<size_t>(a.nbk) + kRowsPerCta) * (dc + 2) * sizeof(double);
  };
  a.dc = a.D;  // whole rows in one pass when they fit, else kDChunk (D % kDChunk == 0)
  if (smem_of(a.dc) > kSmemTarget) a.dc = kDChunk;
  const size_t smem = smem_of(a.dc);
  SAF_CUDA_TRY(cudaFuncSetAttribute(score_topk_kernel<M, RPW>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(smem)));
  dim3 grid(static_cast<unsigned>(BH), (a.nbq + kRowsPerCta - 1) / kRowsPerCta);
  score_topk_kernel<M, RPW><<<grid, 256, smem, st>>>(a);
  return SAF_OK;
}

// Two rows a warp unless that grid leaves SMs without a CTA.  Measured at the
// CogVideoX-2B shape (139 x 139 blocks, B = 2): 4 heads 10.6 us, 30 heads
// 38.3 us.  Four rows a warp (90 KB of shared memory, two CTAs per SM) was
// slower at 15 and 30 heads (30.2 against 20.6 us at 15): with fewer CTAs
// fewer warps hide the chains of dependent fp64 adds.
template <int M>
int32_t launch_score(const SelectArgs& a, int64_t BH, cudaStream_t st) {
  int dev = 0, sms = 0;
  SAF_CUDA_TRY(cudaGetDevice(&dev));
  SAF_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  auto ctas = [&](int rpw) { return BH * ((a.nbq + 8 * rpw - 1) / (8 * rpw)); };
  if (ctas(2) >= sms) return launch_score_rpw<M, 2>(a, BH, st);
  return launch_score_rpw<M, 1>(a, BH, st);
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" size_t saf_pool_topk_workspace_bytes(const saf_tensor4* q, const saf_tensor4* k,
                                                const saf_select_cfg* cfg) {
  if (q == nullptr || k == nullptr || cfg == nullptr || cfg->block_m <= 0 || cfg->block_n <= 0)
    return 0;
  const int nbq = static_cast<int>((q->S + cfg->block_m - 1) / cfg->block_m);
  const int nbk = static_cast<int>((k->S + cfg->block_n - 1) / cfg->block_n);
  return select_layout(q->B * q->H, nbq, nbk, static_cast<int>(q->D)).total;
}

extern "C" int32_t saf_pool_topk(const saf_tensor4* q, const saf_tensor4* k,
                                 const saf_select_cfg* cfg, int32_t* row_ptr, int32_t* col_idx,
                                 uint8_t* mask_out, double* score_out, void* workspace,
                                 size_t workspace_bytes, void* stream) {
  if (cfg == nullptr || row_ptr == nullptr || col_idx == nullptr) return SAF_ERR_ARG;
  int32_t rc;
  if ((rc = check_pool_operand(q)) != SAF_OK) return rc;
  if ((rc = check_pool_operand(k)) != SAF_OK) return rc;
  if (q->dtype != k->dtype) return SAF_ERR_DTYPE;
  if (q->B != k->B || q->H != k->H || q->D != k->D) return SAF_ERR_SHAPE;
  if (cfg->block_m <= 0 || cfg->block_n <= 0 || cfg->topk < 0 || cfg->text_blocks_q < 0 ||
      cfg->text_blocks_k < 0)
    return SAF_ERR_ARG;
  const int64_t nbq64 = (q->S + cfg->block_m - 1) / cfg->block_m;
  const int64_t nbk64 = (k->S + cfg->block_n - 1) / cfg->block_n;
  if (nbk64 > 32 * kMaxM || nbq64 > 1024) return SAF_ERR_SHAPE;
  const int64_t BH = q->B * q->H;
  if (BH * nbq64 * nbk64 >= (int64_t(1) << 31)) return SAF_ERR_SHAPE;  // int32 CSR offsets
  const int nbq = static_cast<int>(nbq64), nbk = static_cast<int>(nbk64);
  const int D = static_cast<int>(q->D);
  if (D % kDChunk != 0) return SAF_ERR_SHAPE;
  const SelectLayout lay = select_layout(BH, nbq, nbk, D);
  if (workspace == nullptr || workspace_bytes < lay.total) return SAF_ERR_WORKSPACE;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return SAF_ERR_WORKSPACE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(q->data)) != SAF_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  double* qbar = reinterpret_cast<double*>(ws + lay.off_qbar);
  double* kbar = reinterpret_cast<double*>(ws + lay.off_kbar);
  if ((rc = pool_dispatch(q, k, cfg->block_m, cfg->block_n, nbq, nbk, qbar, kbar, st)) != SAF_OK)
    return rc;
  SAF_CUDA_TRY(cudaGetLastError());

  SelectArgs a{};
  a.nbq = nbq;
  a.nbk = nbk;
  a.D = D;
  a.topk = cfg->topk;
  a.text_q = cfg->text_blocks_q;
  a.text_k = cfg->text_blocks_k;
  a.force_diag = cfg->force_diag;
  a.forced_inside = cfg->forced_inside_topk;
  a.qbar = qbar;
  a.kbar = kbar;
  a.padded = reinterpret_cast<int32_t*>(ws + lay.off_padded);
  a.counts = reinterpret_cast<int32_t*>(ws + lay.off_counts);
  a.mask_out = mask_out;
  a.score_out = score_out;
  if (nbk <= 160) rc = launch_score<5>(a, BH, st);
  else if (nbk <= 288) rc = launch_score<9>(a, BH, st);
  else rc = launch_score<16>(a, BH, st);
  if (rc != SAF_OK) return rc;
  SAF_CUDA_TRY(cudaGetLastError());
  csr_compact_kernel<<<dim3(static_cast<unsigned>(BH), (nbq + 7) / 8), 256, 0, st>>>(
      nbq, nbk, a.counts, a.padded, row_ptr, col_idx);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

extern "C" int32_t saf_mask_to_csr(const uint8_t* mask, int64_t BH, int32_t nbq, int32_t nbk,
                                   int64_t stride_bh, int64_t stride_row, int32_t* row_ptr,
                                   int32_t* col_idx, void* stream) {
  if (mask == nullptr || row_ptr == nullptr || col_idx == nullptr) return SAF_ERR_ARG;
  if (BH <= 0 || nbq <= 0 || nbk <= 0 || nbq > 16384) return SAF_ERR_SHAPE;
  if (BH * static_cast<int64_t>(nbq) * nbk >= (int64_t(1) << 31)) return SAF_ERR_SHAPE;
  if (stride_row < nbk || stride_bh < 0) return SAF_ERR_STRIDE;
  if (BH > 2147483647) return SAF_ERR_SHAPE;
  DeviceScope dev_scope;
  int32_t rc = dev_scope.bind(mask);
  if (rc != SAF_OK) return rc;
  const size_t smem = (static_cast<size_t>(nbq) + 1) * sizeof(int32_t);
  mask_to_csr_kernel<<<static_cast<unsigned>(BH), 512, smem, static_cast<cudaStream_t>(stream)>>>(
      mask, nbq, nbk, stride_bh, stride_row, row_ptr, col_idx);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

// ---------------------------------------------------------------------------
// Scratch-free block selection.
//
// saf_pool_topk needs a caller-provided workspace.  Some callers cannot
// allocate device memory at the moment they call in: a host process whose
// memory is planned once at start-up and then frozen, a plugin slot that is
// handed only its input and output buffers, or a latency-critical loop that
// must not pay for (or implicitly synchronise on) cudaMalloc.  For them,
// saf_pool_topk_noalloc runs the same kernels with the workspace taken from
// the static array below, which the CUDA module creates on every device that
// loads this library and keeps until the process exits.
//
// The array's name is meaningful only to device code.  Host code must use the
// device address that cudaGetSymbolAddress returns for the current device;
// that lookup happens on the first call for each device (with that device
// current) and is cached.  Nothing in the array has to start at zero: every
// byte the kernels read is written earlier in the same call, so stale data
// from a previous call is harmless.  All calls share the one array, so calls
// whose work overlaps on the GPU (other streams, other host threads) race.
static __device__ __align__(256) unsigned char saf_select_static_scratch[SAF_STATIC_SCRATCH_BYTES];

namespace {
std::mutex g_static_scratch_mu;
void* g_static_scratch_ptr[64] = {nullptr};

int32_t static_scratch_address(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return SAF_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (g_static_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, saf_select_static_scratch) != cudaSuccess || ptr == nullptr) {
      cudaGetLastError();
      return SAF_ERR_CUDA;
    }
    g_static_scratch_ptr[dev] = ptr;
  }
  *out = g_static_scratch_ptr[dev];
  return SAF_OK;
}
}  // namespace

extern "C" int32_t saf_pool_topk_noalloc(const saf_tensor4* q, const saf_tensor4* k,
                                         const saf_select_cfg* cfg, int32_t* row_ptr,
                                         int32_t* col_idx, uint8_t* mask_out, double* score_out,
                                         void* stream) {
  if (q == nullptr || k == nullptr || cfg == nullptr || q->data == nullptr) return SAF_ERR_ARG;
  const size_t need = saf_pool_topk_workspace_bytes(q, k, cfg);
  if (need == 0) return SAF_ERR_ARG;
  if (need > SAF_STATIC_SCRATCH_BYTES) return SAF_ERR_WORKSPACE;  // problem too large for it
  DeviceScope dev_scope;
  int32_t rc = dev_scope.bind(q->data);
  if (rc != SAF_OK) return rc;
  void* scratch = nullptr;
  if ((rc = static_scratch_address(&scratch)) != SAF_OK) return rc;
  return saf_pool_topk(q, k, cfg, row_ptr, col_idx, mask_out, score_out, scratch,
                       SAF_STATIC_SCRATCH_BYTES, stream);
}
