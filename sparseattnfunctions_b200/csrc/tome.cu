// tome.cu -- ToMe bipartite soft matching, merge and unmerge for sm_100a.
//
// Restates special_attentions/utils/merge_unmerge.py:34-154 on the GPU:
//   match  (:99-116) cosine similarity of every src token with every dst
//          token, per src the best dst (node_max, node_idx), src ordered by
//          node_max descending, the first r merged (src_idx -> dst_idx), the
//          rest kept (unm_idx), counter = 1 + number merged into each dst;
//   merge  (:119-135) [unm | dst mean of itself and its merged src];
//   unmerge (:137-154) every token reads its row of the merged sequence.
//
// Exact matching contract (the reference's bf16 scores are tie-dominated):
// cos(a, b) = dot(a, b) / (sqrt(|a|^2) * sqrt(|b|^2)) in fp64 on the input
// values with every dot product summed in one fixed order (products of
// 16-bit values are exact in fp64; lane l of a warp adds the products of
// columns l, l+32, ... in ascending order, then the 32 lane sums are combined
// by an xor butterfly with offsets 16, 8, 4, 2, 1), correctly rounded
// sqrt / mul / div; arg-max ties -> lower dst position, sort ties -> lower
// src position.  Done in three stages so no src x dst score matrix reaches HBM:
//   1. tensor cores (tcgen05, bf16/f16 inputs, fp32 accumulation) score every
//      pair as s~ = dot~ * (1/|b|); each src row keeps its 8 best candidates;
//   2. the candidates are re-scored exactly in fp64.  The fp32 accumulation
//      error of dot~ is below eps * |a| * |b| with eps = 2^-12 (at least 15x
//      the bound (C/16 + 16) * 2^-23 for C <= 2048), so the true best dst has
//      s~ >= s~_top1 - 2 * eps * |a|; when the 8th candidate is below that
//      line the exact winner is among the 8, otherwise the row is re-scanned
//      exactly over all dst;
//   3. a stable radix sort of node_max (descending) orders the src rows.
#include <algorithm>
#include <cub/block/block_exchange.cuh>
#include <cub/block/block_radix_sort.cuh>
#include <cub/device/device_segmented_radix_sort.cuh>

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <type_traits>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kTM = 128;    // src rows per CTA
constexpr int kTN = 256;    // dst columns per MMA tile
constexpr int kTK = 64;     // K chunk: one 128-byte swizzle row of 16-bit values
constexpr int kStages = 4;  // smem ring depth
constexpr int kCand = 8;    // candidates kept per src row
constexpr int kScoreThreads = 384;  // warp 0 TMA, warp 1 MMA, 2-3 idle, 4-11 epilogue
constexpr double kEps = 1.0 / 4096.0;  // accumulation error bound / (|a| |b|)

struct ScoreParams {
  int B, Ns, Nd, Cp;
  const double* na;     // [B, Ns] squared norms of the src rows (fp64)
  const float* rinv_b;  // [B, Nd rounded up to 4] 1 / |b| (fp32; rows 16-byte aligned)
  int32_t* cand_idx;    // [B, Ns, 8]
  float* cand_val;      // [B, Ns, 8]
  unsigned int* status;
  uint64_t budget_ns;
};

constexpr int kResChunks = 4;  // A-resident variant: up to 4 K chunks (C <= 256)

// kRes = false: every stage holds an A and a B chunk (A re-streamed per
// N tile; any C).  kRes = true: the CTA's A rows (at most kResChunks K
// chunks) are loaded once and stay in shared memory, the stages hold B only.
template <bool kRes>
struct ScoreLayoutT {
  static constexpr int kABytes = kTM * kTK * 2;  // 16 KB
  static constexpr int kBBytes = kTN * kTK * 2;  // 32 KB
  static constexpr int kStageBytes = kRes ? kBBytes : kABytes + kBBytes;
  static constexpr int kOffA = 0;
  static constexpr int kOffRing = kRes ? kResChunks * kABytes : 0;
  static constexpr int kOffCand = kOffRing + kStages * kStageBytes;  // [2][128][8] (val, idx)
  static constexpr int kOffBar = kOffCand + 2 * kTM * kCand * 8;
  // full[S], empty[S], acc_full[2], acc_empty[2], drain, xend, a_full,
  // a_empty, xread
  static constexpr int kNumBars = 2 * kStages + 9;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kDynSmem = kOffMisc + 16 + 1024;
};

__device__ __forceinline__ void cand_insert(float (&v)[kCand], int (&ix)[kCand], float s, int j) {
  if (!(s > v[kCand - 1])) return;
  v[kCand - 1] = s;
  ix[kCand - 1] = j;
#pragma unroll
  for (int i = kCand - 1; i > 0; --i) {
    if (v[i] > v[i - 1]) {
      const float tv = v[i];
      v[i] = v[i - 1];
      v[i - 1] = tv;
      const int ti = ix[i];
      ix[i] = ix[i - 1];
      ix[i - 1] = ti;
    }
  }
}

// sc[e] for a runtime e in [0, 32): a 5-level select tree on the bits of e
// (no dynamic register indexing).
__device__ __forceinline__ float pick32(const float (&sc)[32], int e) {
  float l1[16], l2[8], l3[4], l4[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) l1[i] = (e & 1) ? sc[2 * i + 1] : sc[2 * i];
#pragma unroll
  for (int i = 0; i < 8; ++i) l2[i] = (e & 2) ? l1[2 * i + 1] : l1[2 * i];
#pragma unroll
  for (int i = 0; i < 4; ++i) l3[i] = (e & 4) ? l2[2 * i + 1] : l2[2 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) l4[i] = (e & 8) ? l3[2 * i + 1] : l3[2 * i];
  return (e & 16) ? l4[1] : l4[0];
}

// Persistent: one CTA per SM (TMEM: two 256-column accumulators) takes the
// work items (128 src rows of one batch row, batch-row-major) i = blockIdx.x,
// blockIdx.x + gridDim.x, ...; the B ring, the accumulators and the resident
// A carry over from item to item, so an item's first products are made while
// the epilogue still works on the previous item's last tiles.
template <bool kBF16, bool kRes>
__global__ void __launch_bounds__(kScoreThreads, 1)
    tome_score_kernel(const __grid_constant__ CUtensorMap tm_a,
                      const __grid_constant__ CUtensorMap tm_b, const ScoreParams p) {
  using L = ScoreLayoutT<kRes>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mblocks = (p.Ns + kTM - 1) / kTM, n_items = mblocks * p.B;
  const int n_tiles = (p.Nd + kTN - 1) / kTN, k_chunks = p.Cp / kTK;
  const uint32_t ring = smem_u32(smem + L::kOffRing);
  const uint32_t bar0 = smem_u32(smem + L::kOffBar);
  auto bar_full = [&](int s) { return bar0 + 8u * s; };
  auto bar_empty = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto bar_acc_full = [&](int i) { return bar0 + 8u * (2 * kStages + i); };
  auto bar_acc_empty = [&](int i) { return bar0 + 8u * (2 * kStages + 2 + i); };
  const uint32_t bar_drain = bar0 + 8u * (2 * kStages + 4);
  const uint32_t bar_xend = bar0 + 8u * (2 * kStages + 5);
  const uint32_t bar_a = bar0 + 8u * (2 * kStages + 6);        // resident A landed (kRes)
  const uint32_t bar_a_empty = bar0 + 8u * (2 * kStages + 7);  // its products are done (kRes)
  const uint32_t bar_xread = bar0 + 8u * (2 * kStages + 8);    // the half-merge slots were read
  const uint32_t sA = smem_u32(smem + L::kOffA);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full(s), 1);
      mbar_init(bar_empty(s), 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(bar_acc_full(i), 1);
      mbar_init(bar_acc_empty(i), 256);
    }
    mbar_init(bar_drain, 1);
    mbar_init(bar_xend, 256);
    mbar_init(bar_a, 1);
    mbar_init(bar_a_empty, 1);
    mbar_init(bar_xread, 128);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_b);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int issued = 0, items = 0, a_loads = 0;
    if (lane == 0) {
      for (int item = blockIdx.x; item < n_items && !*abort_flag; item += gridDim.x, ++items) {
      const int m0 = (item % mblocks) * kTM, b = item / mblocks;
      if constexpr (kRes) {
        // the previous item's products must be done with the resident A
        if (items > 0 && !mbar_wait(bar_a_empty, (items - 1) & 1, abort_flag, p.status, p.budget_ns)) break;
        mbar_arrive_expect_tx(bar_a, k_chunks * L::kABytes);
        for (int kc = 0; kc < k_chunks; ++kc) tma_load_3d(sA + kc * L::kABytes, &tm_a, bar_a, kc * kTK, m0, b);
        ++a_loads;
      }
      for (int nt = 0; nt < n_tiles; ++nt) {
        for (int kc = 0; kc < k_chunks; ++kc, ++issued) {
          const int s = issued % kStages;
          const uint32_t ph = (issued / kStages) & 1;
          if (!mbar_wait(bar_empty(s), ph ^ 1, abort_flag, p.status, p.budget_ns)) break;
          const uint32_t st = ring + s * L::kStageBytes;
          mbar_arrive_expect_tx(bar_full(s), L::kStageBytes);
          if constexpr (kRes) {
            tma_load_3d(st, &tm_b, bar_full(s), kc * kTK, nt * kTN, b);
          } else {
            tma_load_3d(st, &tm_a, bar_full(s), kc * kTK, m0, b);
            tma_load_3d(st + L::kABytes, &tm_b, bar_full(s), kc * kTK, nt * kTN, b);
          }
        }
        if (*abort_flag) break;
      }
      }
      // drain: wait for the last load of every stage (and the resident A)
      if constexpr (kRes) {
        if (a_loads > 0) mbar_drain(bar_a, (a_loads - 1) & 1, p.status);
      }
      for (int s = 0; s < kStages && s < issued; ++s) {
        const int last = s + ((issued - 1 - s) / kStages) * kStages;
        mbar_drain(bar_full(s), (last / kStages) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16(kTM, kTN, kBF16, false, false);
      int used = 0, ntg = 0;  // K chunks consumed, tiles made (all items)
      bool ok = true;
      for (int item = blockIdx.x, items = 0; item < n_items && ok; item += gridDim.x, ++items) {
      if constexpr (kRes) ok = mbar_wait(bar_a, items & 1, abort_flag, p.status, p.budget_ns);
      for (int nt = 0; nt < n_tiles && ok; ++nt, ++ntg) {
        const int buf = ntg & 1;
        if (!mbar_wait(bar_acc_empty(buf), ((ntg >> 1) & 1) ^ 1, abort_flag, p.status,
                       p.budget_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + buf * kTN;
        for (int kc = 0; kc < k_chunks; ++kc, ++used) {
          const int s = used % kStages;
          if (!mbar_wait(bar_full(s), (used / kStages) & 1, abort_flag, p.status, p.budget_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = ring + s * L::kStageBytes;
          const uint32_t a_chunk = kRes ? sA + kc * L::kABytes : st;
          const uint32_t b_chunk = kRes ? st : st + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kTK / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(a_chunk + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(b_chunk + kk * 32, 16, 1024);
            tc_mma_ss(acc, ad, bd, kIdesc, (kc > 0 || kk > 0) ? 1u : 0u);
          }
          tc_commit(bar_empty(s));
        }
        if (ok) tc_commit(bar_acc_full(buf));
      }
      // the resident A is free once this item's products are done
      if constexpr (kRes) {
        if (ok) tc_commit(bar_a_empty);
      }
      }
      tc_commit(bar_drain);
      mbar_drain(bar_drain, 0, p.status);
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3, chalf = (warp - 4) >> 2;
    const int row = quarter * 32 + lane;
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    int ntg = 0;  // tiles taken (all items)
    for (int item = blockIdx.x, items = 0; item < n_items && ok; item += gridDim.x, ++items) {
    const int m0 = (item % mblocks) * kTM, b = item / mblocks;
    const float* rinv = p.rinv_b + static_cast<int64_t>(b) * ((p.Nd + 3) & ~3);
    // Candidates of this thread's half of the row: every column whose score
    // came within tau of the running maximum when it was seen (the only
    // columns that can hold the exact best, as each score is within tau / 2
    // of its exact value), at most kCand of them, in descending order.  A
    // column still within tau that does not fit sets `ovf`: the row then
    // takes the exact full scan.  tau is widened by 1/256 so that fp32
    // rounding of the comparisons cannot drop a candidate.
    const double na_row = m0 + row < p.Ns ? p.na[static_cast<int64_t>(b) * p.Ns + m0 + row] : 0.0;
    const float tau = static_cast<float>(2.0 * kEps * sqrt(na_row) * (1.0 + 1.0 / 256.0));
    float cv[kCand];
    int ci[kCand];
#pragma unroll
    for (int i = 0; i < kCand; ++i) {
      cv[i] = -INFINITY;
      ci[i] = -1;
    }
    float run_max = -INFINITY;
    bool ovf = false;
    auto add = [&](float sv, int j, float thr) {
      if (ci[kCand - 1] >= 0 && fminf(sv, cv[kCand - 1]) >= thr) ovf = true;
      cand_insert(cv, ci, sv, j);
    };
    float4 rv_next[8];
    if (chalf * (kTN / 2) + 32 <= p.Nd) {
#pragma unroll
      for (int i = 0; i < 8; ++i) rv_next[i] = __ldg(reinterpret_cast<const float4*>(rinv + chalf * (kTN / 2)) + i);
    }
    for (int nt = 0; nt < n_tiles; ++nt, ++ntg) {
      const int buf = ntg & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar_acc_full(buf), (ntg >> 1) & 1, abort_flag,
                                              p.status, p.budget_ns))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const int col0 = nt * kTN + chalf * (kTN / 2);
#pragma unroll 1
      for (int c = 0; c < kTN / 2 / 32; ++c) {
        const int jc = col0 + c * 32;
        // this chunk's 1/|b| (prefetched one chunk ahead); the next chunk's
        // loads are issued before this chunk's TMEM load
        float4 rv[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rv[i] = rv_next[i];
        {
          const int jn = c + 1 < kTN / 2 / 32 ? jc + 32 : (nt + 1) * kTN + chalf * (kTN / 2);
          if (jn + 32 <= p.Nd) {
#pragma unroll
            for (int i = 0; i < 8; ++i) rv_next[i] = __ldg(reinterpret_cast<const float4*>(rinv + jn) + i);
          }
        }
        uint32_t r[32];
        tmem_ld32(tmem + lane_addr + buf * kTN + chalf * (kTN / 2) + c * 32, r);
        tmem_wait_ld(r);
        if (c == kTN / 2 / 32 - 1) {
          tc_fence_before();
          mbar_arrive(bar_acc_empty(buf));
        }
        // scores of the chunk (1/|b| shared by every lane of the warp);
        // columns past Nd score -inf
        float sc[32];
        if (jc + 32 <= p.Nd) {
#pragma unroll
          for (int e = 0; e < 32; e += 4) {
            const float4 q = rv[e / 4];
            const f2 a = mul2(mk2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), mk2(q.x, q.y));
            const f2 b2 = mul2(mk2(__uint_as_float(r[e + 2]), __uint_as_float(r[e + 3])), mk2(q.z, q.w));
            sc[e] = lo2(a);
            sc[e + 1] = hi2(a);
            sc[e + 2] = lo2(b2);
            sc[e + 3] = hi2(b2);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e)
            sc[e] = jc + e < p.Nd ? __uint_as_float(r[e]) * __ldg(rinv + jc + e) : -INFINITY;
        }
        float m4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) m4[i] = fmax3(sc[8 * i], sc[8 * i + 1], sc[8 * i + 2]);
#pragma unroll
        for (int i = 0; i < 4; ++i) m4[i] = fmax3(m4[i], sc[8 * i + 3], sc[8 * i + 4]);
#pragma unroll
        for (int i = 0; i < 4; ++i) m4[i] = fmax3(m4[i], sc[8 * i + 5], sc[8 * i + 6]);
#pragma unroll
        for (int i = 0; i < 4; ++i) m4[i] = fmaxf(m4[i], sc[8 * i + 7]);
        const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        // most chunks hold nothing within tau of the running maximum
        if (mx >= run_max - tau) {
          run_max = fmaxf(run_max, mx);
          const float thr = run_max - tau;
          // bit e = (sc[e] >= thr): the sign bits of sc - thr, gathered by
          // funnel shifts in four independent chains.  The sign is exact
          // (a difference of two floats rounds to zero only when it is zero),
          // and -thr + 0 is never -0, so sc = -0 against thr = 0 gives +0.
          uint32_t nb[4] = {0u, 0u, 0u, 0u};
          const float nthr = -thr + 0.0f;
          const f2 thr2 = mk2(nthr, nthr);
#pragma unroll
          for (int e = 30; e >= 0; e -= 2) {
            const f2 d = add2(mk2(sc[e], sc[e + 1]), thr2);
            const int g = (e >> 3) & 3;
            nb[g] = __funnelshift_l(__float_as_uint(lo2(d)), __funnelshift_l(__float_as_uint(hi2(d)), nb[g], 1), 1);
          }
          uint32_t mask = ~(nb[0] | (nb[1] << 8) | (nb[2] << 16) | (nb[3] << 24));
          if ((mask & (mask - 1)) == 0) {
            add(mx, jc + __ffs(mask) - 1, thr);  // the chunk maximum, usually alone
          } else if (__popc(mask) <= 4) {
            // a few columns within tau: in ascending column order
            while (mask) {
              const int e = __ffs(mask) - 1;
              mask &= mask - 1;
              add(pick32(sc, e), jc + e, thr);
            }
          } else {
            // many (near-duplicate dst rows): every column, predicated
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if ((mask >> e) & 1u) add(sc[e], jc + e, thr);
          }
        }
      }
    }
    // merge the two column halves of every row
    float2* cand = reinterpret_cast<float2*>(smem + L::kOffCand);
    if (chalf == 1) {
      // the slots are free once the other half has read the previous item's
      if (ok && items > 0 &&
          !__all_sync(0xffffffffu, mbar_wait(bar_xread, (items - 1) & 1, abort_flag, p.status, p.budget_ns)))
        ok = false;
      if (ok) {
#pragma unroll
        for (int i = 0; i < kCand; ++i)
          cand[(kTM + row) * kCand + i] = make_float2(cv[i], __int_as_float(ci[i]));
        cand[row * kCand] = make_float2(run_max, __int_as_float(ovf ? 1 : 0));
      }
    }
    mbar_arrive(bar_xend);
    const bool have = ok && __all_sync(0xffffffffu, mbar_wait(bar_xend, items & 1, abort_flag, p.status,
                                                               p.budget_ns));
    if (!have) ok = false;
    if (have && chalf == 0 && m0 + row < p.Ns && !*abort_flag) {
      const float2 hdr = cand[row * kCand];
      run_max = fmaxf(run_max, hdr.x);
      ovf = ovf || __float_as_int(hdr.y) != 0;
      const float thr = run_max - tau;
#pragma unroll
      for (int i = 0; i < kCand; ++i) {
        const float2 o = cand[(kTM + row) * kCand + i];
        if (__float_as_int(o.y) >= 0 && o.x >= thr) add(o.x, __float_as_int(o.y), thr);
      }
      // an incomplete row is marked by candidate index -2 in the last slot
      if (ovf) ci[kCand - 1] = -2;
      const int64_t base = (static_cast<int64_t>(b) * p.Ns + m0 + row) * kCand;
#pragma unroll
      for (int i = 0; i < kCand; ++i) {
        p.cand_idx[base + i] = ci[i];
        p.cand_val[base + i] = cv[i];
      }
    }
    if (chalf == 0) mbar_arrive(bar_xread);
    }  // items
  }
  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------------------
// gather + norms: one warp per gathered row.
template <typename T>
__device__ __forceinline__ double ld_f64(const T* p) {
  if constexpr (sizeof(T) == 2) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) return static_cast<double>(__bfloat162float(*p));
    else return static_cast<double>(__half2float(*p));
  } else {
    return static_cast<double>(*p);
  }
}

struct GatherParams {
  const void* metric;
  int64_t sb, sn;  // element strides of metric [B, N, C]
  int B, N, C, Cp;
  const int32_t* idx;  // [n_rows] token indices
  int n_rows;
  void* out;           // [B, n_rows, Cp] 16-bit
  double* sqnorm;      // [B, n_rows]
  float* rinv;         // [B, n_rows rounded up to 4] or null
  unsigned int* status;
};

// Four gathered rows per warp (independent loads in flight); each row's
// squared norm keeps the contract's order (lane l: columns l, l + 32, ...
// ascending, then the xor butterfly).
constexpr int kGatherRows = 4;

template <typename T>
__global__ void __launch_bounds__(256) tome_gather_kernel(const GatherParams g) {
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int r0 = w * kGatherRows;
  if (r0 >= g.n_rows) return;
  const T* src[kGatherRows];
  T* dst[kGatherRows];
  bool ok[kGatherRows];
  double acc[kGatherRows];
#pragma unroll
  for (int r = 0; r < kGatherRows; ++r) {
    const int row = min(r0 + r, g.n_rows - 1);
    int tok = g.idx[row];
    if (tok < 0 || tok >= g.N) {
      if (lane == 0 && r0 + r < g.n_rows) atomicOr(g.status, SAF_DEV_BADINDEX);
      tok = -1;
    }
    ok[r] = tok >= 0;
    src[r] = static_cast<const T*>(g.metric) + static_cast<int64_t>(b) * g.sb +
             static_cast<int64_t>(tok < 0 ? 0 : tok) * g.sn;
    dst[r] = static_cast<T*>(g.out) + (static_cast<int64_t>(b) * g.n_rows + row) * g.Cp;
    acc[r] = 0.0;
  }
  // two columns per lane and row loaded before any store (eight loads in flight)
  for (int c0 = lane; c0 < g.Cp; c0 += 64) {
    T v[2][kGatherRows];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = c0 + 32 * u;
#pragma unroll
      for (int r = 0; r < kGatherRows; ++r) v[u][r] = (c < g.C && ok[r]) ? src[r][c] : T(0.f);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int c = c0 + 32 * u;
      if (c >= g.Cp) break;
#pragma unroll
      for (int r = 0; r < kGatherRows; ++r) {
        if (r0 + r < g.n_rows) dst[r][c] = v[u][r];
        const double d = ld_f64(&v[u][r]);
        acc[r] = fma(d, d, acc[r]);  // products of 16-bit values are exact in fp64
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kGatherRows; ++r) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) acc[r] += __shfl_xor_sync(0xffffffffu, acc[r], off);
    const int row = r0 + r;
    if (lane == 0 && row < g.n_rows) {
      g.sqnorm[static_cast<int64_t>(b) * g.n_rows + row] = acc[r];
      if (g.rinv)
        g.rinv[static_cast<int64_t>(b) * ((g.n_rows + 3) & ~3) + row] = static_cast<float>(1.0 / sqrt(acc[r]));
    }
  }
}

// ---------------------------------------------------------------------------
// exact re-score: one warp per src row.
struct ExactParams {
  const void* A;        // [B, Ns, Cp] 16-bit
  const void* Bm;       // [B, Nd, Cp] 16-bit
  const double* na;     // [B, Ns]
  const double* nb;     // [B, Nd]
  const int32_t* cand_idx;
  const float* cand_val;
  int B, Ns, Nd, Cp;
  double* node_max;     // [B, Ns]
  int32_t* node_idx;    // [B, Ns]
};

// Eight columns per lane are loaded before they are summed, so a lane has
// 16 loads in flight instead of two (a zero pad past Cp adds +0 and leaves
// every partial sum unchanged).
template <typename T>
__device__ __forceinline__ double exact_dot(const T* a, const T* bb, int Cp, int lane) {
  double acc = 0.0;
  for (int c0 = lane; c0 < Cp; c0 += 32 * 8) {
    double av[8], bv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int c = c0 + 32 * i;
      av[i] = c < Cp ? ld_f64(a + c) : 0.0;
      bv[i] = c < Cp ? ld_f64(bb + c) : 0.0;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) acc = fma(av[i], bv[i], acc);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return acc;  // the contract's summation order (see the file header)
}

// Columns of a row each lane holds in the short-row path (Cp <= 256).
constexpr int kExactCols = 8;

// Dot of this lane's a columns (held) with row b, in the contract's order:
// lane l sums columns l, l+32, ... ascending, then the butterfly below.
template <typename T>
__device__ __forceinline__ double held_dot(const T (&av)[kExactCols], const T (&bv)[kExactCols]) {
  double acc = 0.0;
#pragma unroll
  for (int i = 0; i < kExactCols; ++i) acc = fma(ld_f64(&av[i]), ld_f64(&bv[i]), acc);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, off);
  return acc;
}

// One warp per src row (rows differ a thousandfold in cost, so CTAs of eight
// rows are handed out by the hardware rather than split up front).  A short
// row (Cp <= 256) takes two dependent memory round trips: its a row, norm
// and candidate list together, then the dst rows and norms of the
// candidates to re-score, two at a time (four at a time in the full scan).
// The winner is the largest exact cosine, ties to the lower dst index, so
// the order the candidates are scored in does not matter.
template <typename T, bool kShort>
__global__ void __launch_bounds__(256, kShort ? 4 : 3) tome_exact_kernel(const ExactParams e) {
  const int lane = threadIdx.x & 31;
  constexpr bool short_rows = kShort;  // Cp <= 32 * kExactCols
  const int b = blockIdx.y;
  const int i = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  if (i >= e.Ns) return;
  const int64_t ri = static_cast<int64_t>(b) * e.Ns + i;
  const T* a = static_cast<const T*>(e.A) + ri * e.Cp;
  // independent loads first
  const double na = e.na[ri];
  const float cvl = lane < kCand ? e.cand_val[ri * kCand + lane] : -INFINITY;
  const int cil = lane < kCand ? e.cand_idx[ri * kCand + lane] : -1;
  T av[kExactCols];  // 16-bit values; a zero pad adds +0 and changes no sum
#pragma unroll
  for (int q = 0; q < kExactCols; ++q) {
    const int c = lane + 32 * q;
    av[q] = (short_rows && c < e.Cp) ? a[c] : T(0.f);
  }
  const double sa = __dsqrt_rn(na);
  const double tau = 2.0 * kEps * sa;  // in units of s~ = dot * (1/|b|)
  const float cv0 = __shfl_sync(0xffffffffu, cvl, 0);
  // The score kernel kept every column within tau of the row's maximum
  // unless it marked the row incomplete (index -2 in the last slot).
  const bool complete = e.Nd <= kCand || __shfl_sync(0xffffffffu, cil, kCand - 1) != -2;
  // A candidate can be the exact best only if its tensor-core score is
  // within tau of the top one (each score is within tau / 2 of its exact
  // value).
  const float keep_above = static_cast<float>(static_cast<double>(cv0) - tau * (1.0 + 1.0 / 256.0));
  double best = -INFINITY;
  int bj = 0x7fffffff;
  auto take = [&](double d, int j) {
    const double cs = __ddiv_rn(d, __dmul_rn(sa, __dsqrt_rn(e.nb[static_cast<int64_t>(b) * e.Nd + j])));
    if (cs > best || (cs == best && j < bj)) {
      best = cs;
      bj = j;
    }
  };
  const T* bbase = static_cast<const T*>(e.Bm) + static_cast<int64_t>(b) * e.Nd * e.Cp;
  if constexpr (kShort) {
    if (!complete) {  // every dst, four at a time
#pragma unroll 1
      for (int j0 = 0; j0 < e.Nd; j0 += 4) {
        T bv[4][kExactCols];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const T* bj_row = bbase + static_cast<int64_t>(min(j0 + u, e.Nd - 1)) * e.Cp;
#pragma unroll
          for (int q = 0; q < kExactCols; ++q) {
            const int c = lane + 32 * q;
            bv[u][q] = c < e.Cp ? bj_row[c] : T(0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + u < e.Nd) take(held_dot<T>(av, bv[u]), j0 + u);
      }
    } else {
    uint32_t m = __ballot_sync(0xffffffffu, lane < kCand && lane < e.Nd && cil >= 0 &&
                                                (lane == 0 || cvl >= keep_above));
    while (m != 0u) {
      const int k0 = __ffs(m) - 1;
      m &= m - 1u;
      const int k1 = m != 0u ? __ffs(m) - 1 : k0;
      if (m != 0u) m &= m - 1u;
      const int j0 = __shfl_sync(0xffffffffu, cil, k0), j1 = __shfl_sync(0xffffffffu, cil, k1);
      const T* b0 = bbase + static_cast<int64_t>(j0) * e.Cp;
      const T* b1 = bbase + static_cast<int64_t>(j1) * e.Cp;
      T bv0[kExactCols], bv1[kExactCols];
#pragma unroll
      for (int q = 0; q < kExactCols; ++q) {
        const int c = lane + 32 * q;
        bv0[q] = c < e.Cp ? b0[c] : T(0.f);
        bv1[q] = (k1 != k0 && c < e.Cp) ? b1[c] : T(0.f);
      }
      take(held_dot<T>(av, bv0), j0);
      if (k1 != k0) take(held_dot<T>(av, bv1), j1);
    }
    }
  } else {
    auto consider = [&](int j) { take(exact_dot(a, bbase + static_cast<int64_t>(j) * e.Cp, e.Cp, lane), j); };
    if (complete) {
#pragma unroll 1
      for (int k = 0; k < kCand && k < e.Nd; ++k) {
        const int j = __shfl_sync(0xffffffffu, cil, k);
        const float cvk = __shfl_sync(0xffffffffu, cvl, k);
        if (j >= 0 && (k == 0 || cvk >= keep_above)) consider(j);
      }
    } else {
#pragma unroll 1
      for (int j = 0; j < e.Nd; ++j) consider(j);
    }
  }
  if (lane == 0) {
    e.node_max[ri] = best;
    e.node_idx[ri] = bj;
  }
}

// ---------------------------------------------------------------------------
// Per-segment stable radix sorts with one CTA per batch row, the whole
// segment on chip (segments up to kSortCap items; larger ones take the
// device-wide segmented sort).  Items are read and written in a striped
// arrangement (coalesced) and exchanged to/from the blocked arrangement whose
// order defines stability.  Padding keys sort last (-inf for descending fp64,
// all ones in the sorted bits for ascending int32) and stability keeps them
// behind real keys of the same value.
constexpr int kSortThreads = 512;
constexpr int kSortCap = kSortThreads * 32;  // 16384

template <typename K, bool kDesc, int kItems>
__global__ void __launch_bounds__(kSortThreads) tome_block_sort_kernel(const K* __restrict__ keys,
                                                                       const int32_t* __restrict__ vals,
                                                                       K* __restrict__ keys_out,
                                                                       int32_t* __restrict__ vals_out, int n,
                                                                       int end_bit) {
  using Sort = cub::BlockRadixSort<K, kSortThreads, kItems, int32_t>;
  using ExK = cub::BlockExchange<K, kSortThreads, kItems>;
  using ExV = cub::BlockExchange<int32_t, kSortThreads, kItems>;
  union Smem {
    typename Sort::TempStorage sort;
    typename ExK::TempStorage exk;
    typename ExV::TempStorage exv;
  };
  extern __shared__ __align__(16) uint8_t sort_smem[];
  Smem& sm = *reinterpret_cast<Smem*>(sort_smem);
  const int64_t base = static_cast<int64_t>(blockIdx.x) * n;
  const int tid = threadIdx.x;
  K k[kItems];
  int32_t v[kItems];
  const K pad = kDesc ? static_cast<K>(-INFINITY) : static_cast<K>(0x7fffffff);
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int idx = i * kSortThreads + tid;
    k[i] = idx < n ? keys[base + idx] : pad;
  }
  ExK(sm.exk).StripedToBlocked(k);
  __syncthreads();
  if (vals) {
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int idx = i * kSortThreads + tid;
      v[i] = idx < n ? vals[base + idx] : 0x7fffffff;
    }
    ExV(sm.exv).StripedToBlocked(v);
    __syncthreads();
  } else {
#pragma unroll
    for (int i = 0; i < kItems; ++i) v[i] = tid * kItems + i;
  }
  if constexpr (kDesc)
    Sort(sm.sort).SortDescendingBlockedToStriped(k, v, 0, end_bit);
  else
    Sort(sm.sort).SortBlockedToStriped(k, v, 0, end_bit);
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int idx = i * kSortThreads + tid;
    if (idx < n) {
      vals_out[base + idx] = v[i];
      if (keys_out) keys_out[base + idx] = k[i];
    }
  }
}

template <typename K, bool kDesc, int kItems>
cudaError_t block_sort_items(const K* keys, const int32_t* vals, K* keys_out, int32_t* vals_out, int B, int n,
                             int end_bit, cudaStream_t st) {
  constexpr int smem = static_cast<int>(
      std::max({sizeof(typename cub::BlockRadixSort<K, kSortThreads, kItems, int32_t>::TempStorage),
                sizeof(typename cub::BlockExchange<K, kSortThreads, kItems>::TempStorage),
                sizeof(typename cub::BlockExchange<int32_t, kSortThreads, kItems>::TempStorage)}));
  cudaError_t e = cudaFuncSetAttribute(tome_block_sort_kernel<K, kDesc, kItems>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  tome_block_sort_kernel<K, kDesc, kItems><<<B, kSortThreads, smem, st>>>(keys, vals, keys_out, vals_out, n,
                                                                          end_bit);
  return cudaGetLastError();
}

// Sorts B segments of n items each (n <= kSortCap) with the smallest
// per-thread item count that holds a segment.
template <typename K, bool kDesc>
cudaError_t block_sort(const K* keys, const int32_t* vals, K* keys_out, int32_t* vals_out, int B, int n,
                       int end_bit, cudaStream_t st) {
  if (n <= kSortThreads * 8) return block_sort_items<K, kDesc, 8>(keys, vals, keys_out, vals_out, B, n, end_bit, st);
  if (n <= kSortThreads * 16)
    return block_sort_items<K, kDesc, 16>(keys, vals, keys_out, vals_out, B, n, end_bit, st);
  if (n <= kSortThreads * 24)
    return block_sort_items<K, kDesc, 24>(keys, vals, keys_out, vals_out, B, n, end_bit, st);
  return block_sort_items<K, kDesc, 32>(keys, vals, keys_out, vals_out, B, n, end_bit, st);
}

// ---------------------------------------------------------------------------
// plan finalisation
struct FinalParams {
  int B, Ns, Nd, N, r;
  const int32_t* order;        // [B, Ns] src positions sorted by node_max desc
  const int32_t* node_idx;     // [B, Ns]
  const int32_t* a_idx;        // [Ns]
  const int32_t* b_idx;        // [Nd]
  int32_t* unm_idx;            // [B, Ns - r]
  int32_t* src_idx;            // [B, r]
  int32_t* dst_idx;            // [B, r]
  int32_t* dst_key;            // [B, r] (sort input: dst of the k-th merged src)
  int32_t* dst_val;            // [B, r] (sort input: its src position)
  int32_t* token_map;          // [B, N] or null
};

__global__ void tome_final_kernel(const FinalParams f) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
  const int64_t bo = static_cast<int64_t>(b);
  const int unm_len = f.Ns - f.r;
  if (k < f.Nd && f.token_map) f.token_map[bo * f.N + f.b_idx[k]] = unm_len + k;
  if (k >= f.Ns) return;
  const int s = f.order[bo * f.Ns + k];
  if (k < f.r) {
    const int d = f.node_idx[bo * f.Ns + s];
    f.src_idx[bo * f.r + k] = s;
    f.dst_idx[bo * f.r + k] = d;
    f.dst_key[bo * f.r + k] = d;
    f.dst_val[bo * f.r + k] = s;
    if (f.token_map) f.token_map[bo * f.N + f.a_idx[s]] = unm_len + d;
  } else {
    f.unm_idx[bo * unm_len + (k - f.r)] = s;
    if (f.token_map) f.token_map[bo * f.N + f.a_idx[s]] = k - f.r;
  }
}

// dst_ptr[b, j] = first position of dst j in the dst-sorted merged list;
// counter = 1 + count; log_count = log(counter).
__global__ void tome_dstptr_kernel(int B, int Nd, int r, const int32_t* __restrict__ keys_sorted,
                                   int32_t* __restrict__ dst_ptr, int32_t* __restrict__ counter,
                                   float* __restrict__ log_count) {
  const int j = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
  if (j > Nd) return;
  const int32_t* kk = keys_sorted + static_cast<int64_t>(b) * r;
  int lo = 0, hi = r;  // lower_bound(j)
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (kk[mid] < j) lo = mid + 1;
    else hi = mid;
  }
  dst_ptr[static_cast<int64_t>(b) * (Nd + 1) + j] = lo;
  if (j < Nd) {
    int lo2 = lo, hi2 = r;  // lower_bound(j + 1)
    while (lo2 < hi2) {
      const int mid = (lo2 + hi2) >> 1;
      if (kk[mid] < j + 1) lo2 = mid + 1;
      else hi2 = mid;
    }
    const int c = 1 + (lo2 - lo);
    counter[static_cast<int64_t>(b) * Nd + j] = c;
    if (log_count) log_count[static_cast<int64_t>(b) * Nd + j] = logf(static_cast<float>(c));
  }
}

__global__ void tome_offsets_kernel(int B, int n, int* __restrict__ off) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i <= B) off[i] = i * n;
}

__global__ void tome_iota_kernel(int B, int n, int32_t* __restrict__ v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x, b = blockIdx.y;
  if (i < n) v[static_cast<int64_t>(b) * n + i] = i;
}

// ---------------------------------------------------------------------------
// merge / unmerge: one warp per output row.
struct RowCopyParams {
  const void* x;
  void* out;
  int64_t x_sb, x_sn, o_sb, o_sn;  // element strides ([B, rows, C])
  int B, C, text;                  // text rows copied unchanged
  int Ns, Nd, r, N;
  const int32_t* a_idx;
  const int32_t* b_idx;
  const int32_t* unm_idx;   // [B, Ns - r]
  const int32_t* counter;   // [B, Nd]
  const int32_t* dst_ptr;   // [B, Nd + 1]
  const int32_t* dst_src;   // [B, r]
  const int32_t* token_map; // [B, N]
};

template <typename T>
__device__ __forceinline__ float to_f(T v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __bfloat162float(v);
  else if constexpr (std::is_same<T, __half>::value) return __half2float(v);
  else return v;
}
template <typename T>
__device__ __forceinline__ T from_f(float v) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(v);
  else if constexpr (std::is_same<T, __half>::value) return __float2half_rn(v);
  else return v;
}

template <typename T>
__global__ void __launch_bounds__(256) tome_merge_kernel(const RowCopyParams q) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  const int unm_len = q.Ns - q.r;
  const int out_rows = q.text + unm_len + q.Nd;
  if (row >= out_rows) return;
  const T* xb = static_cast<const T*>(q.x) + static_cast<int64_t>(b) * q.x_sb;
  T* ob = static_cast<T*>(q.out) + static_cast<int64_t>(b) * q.o_sb + static_cast<int64_t>(row) * q.o_sn;
  const int64_t bo = b;
  if (row < q.text || row < q.text + unm_len) {
    const int src_row = row < q.text ? row : q.text + q.a_idx[q.unm_idx[bo * unm_len + row - q.text]];
    const T* xs = xb + static_cast<int64_t>(src_row) * q.x_sn;
    for (int c = lane; c < q.C; c += 32) ob[c] = xs[c];
    return;
  }
  // dst row: (x_dst + sum of merged src, in ascending merge order) / counter
  const int j = row - q.text - unm_len;
  const T* xd = xb + static_cast<int64_t>(q.text + q.b_idx[j]) * q.x_sn;
  const int p0 = q.dst_ptr[bo * (q.Nd + 1) + j], p1 = q.dst_ptr[bo * (q.Nd + 1) + j + 1];
  const float inv = 1.f / static_cast<float>(q.counter[bo * q.Nd + j]);
  for (int c = lane; c < q.C; c += 32) {
    float acc = to_f(xd[c]);
    for (int t = p0; t < p1; ++t) {
      const int s = q.dst_src[bo * q.r + t];
      acc += to_f(xb[static_cast<int64_t>(q.text + q.a_idx[s]) * q.x_sn + c]);
    }
    ob[c] = from_f<T>(acc * inv);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) tome_unmerge_kernel(const RowCopyParams q) {
  const int row = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.y;
  if (row >= q.text + q.N) return;
  const int src_row = row < q.text ? row : q.text + q.token_map[static_cast<int64_t>(b) * q.N + row - q.text];
  const T* xs = static_cast<const T*>(q.x) + static_cast<int64_t>(b) * q.x_sb + static_cast<int64_t>(src_row) * q.x_sn;
  T* ob = static_cast<T*>(q.out) + static_cast<int64_t>(b) * q.o_sb + static_cast<int64_t>(row) * q.o_sn;
  if ((q.C * sizeof(T)) % 16 == 0 && (reinterpret_cast<uintptr_t>(xs) & 15) == 0 &&
      (reinterpret_cast<uintptr_t>(ob) & 15) == 0) {
    const int nv = q.C * static_cast<int>(sizeof(T)) / 16;
    for (int c = lane; c < nv; c += 32) reinterpret_cast<uint4*>(ob)[c] = reinterpret_cast<const uint4*>(xs)[c];
  } else {
    for (int c = lane; c < q.C; c += 32) ob[c] = xs[c];
  }
}

// Vectorised forms: one thread per 16-byte chunk of an output row, so rows
// narrower than a warp's 512 bytes (the per-head D = 64 layout of merged
// attention) still keep every lane busy.  Used when every row start is
// 16-byte aligned; the warp-per-row kernels above cover the rest.
template <typename T>
struct Vec16 {
  static constexpr int kN = 16 / static_cast<int>(sizeof(T));
};

template <typename T>
__device__ __forceinline__ void acc16(float (&a)[Vec16<T>::kN], const uint4 v) {
  const T* e = reinterpret_cast<const T*>(&v);
#pragma unroll
  for (int i = 0; i < Vec16<T>::kN; ++i) a[i] += to_f(e[i]);
}

template <typename T>
__global__ void __launch_bounds__(256) tome_merge_vec_kernel(const RowCopyParams q, const int chunks,
                                                             const int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int row = static_cast<int>(idx / chunks), ch = static_cast<int>(idx - static_cast<int64_t>(row) * chunks);
  const int b = blockIdx.y;
  const int64_t bo = b;
  const int unm_len = q.Ns - q.r;
  const T* xb = static_cast<const T*>(q.x) + bo * q.x_sb;
  uint4* op = reinterpret_cast<uint4*>(static_cast<T*>(q.out) + bo * q.o_sb + static_cast<int64_t>(row) * q.o_sn) + ch;
  if (row < q.text + unm_len) {
    const int src_row = row < q.text ? row : q.text + q.a_idx[q.unm_idx[bo * unm_len + row - q.text]];
    *op = __ldg(reinterpret_cast<const uint4*>(xb + static_cast<int64_t>(src_row) * q.x_sn) + ch);
    return;
  }
  // dst row: (x_dst + merged src rows in ascending merge order) / counter, in fp32
  constexpr int kN = Vec16<T>::kN;
  const int j = row - q.text - unm_len;
  float a[kN];
#pragma unroll
  for (int i = 0; i < kN; ++i) a[i] = 0.f;
  acc16<T>(a, __ldg(reinterpret_cast<const uint4*>(xb + static_cast<int64_t>(q.text + q.b_idx[j]) * q.x_sn) + ch));
  const int p0 = q.dst_ptr[bo * (q.Nd + 1) + j], p1 = q.dst_ptr[bo * (q.Nd + 1) + j + 1];
  for (int t = p0; t < p1; ++t) {
    const int s = q.dst_src[bo * q.r + t];
    acc16<T>(a, __ldg(reinterpret_cast<const uint4*>(xb + static_cast<int64_t>(q.text + q.a_idx[s]) * q.x_sn) + ch));
  }
  const float inv = 1.f / static_cast<float>(q.counter[bo * q.Nd + j]);
  uint4 o;
  T* oe = reinterpret_cast<T*>(&o);
#pragma unroll
  for (int i = 0; i < kN; ++i) oe[i] = from_f<T>(a[i] * inv);
  *op = o;
}

template <typename T>
__global__ void __launch_bounds__(256) tome_unmerge_vec_kernel(const RowCopyParams q, const int chunks,
                                                               const int64_t total) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  const int row = static_cast<int>(idx / chunks), ch = static_cast<int>(idx - static_cast<int64_t>(row) * chunks);
  const int64_t bo = blockIdx.y;
  const int src_row = row < q.text ? row : q.text + q.token_map[bo * q.N + row - q.text];
  const uint4* xs = reinterpret_cast<const uint4*>(static_cast<const T*>(q.x) + bo * q.x_sb +
                                                   static_cast<int64_t>(src_row) * q.x_sn) + ch;
  uint4* op = reinterpret_cast<uint4*>(static_cast<T*>(q.out) + bo * q.o_sb + static_cast<int64_t>(row) * q.o_sn) + ch;
  *op = __ldg(xs);
}

// True when every row of x and out starts on a 16-byte boundary and C fills whole 16-byte chunks.
bool rows_vec16(const RowCopyParams& q, size_t elem) {
  const int64_t v = 16 / static_cast<int64_t>(elem);
  return (q.C * elem) % 16 == 0 && (reinterpret_cast<uintptr_t>(q.x) & 15) == 0 &&
         (reinterpret_cast<uintptr_t>(q.out) & 15) == 0 && q.x_sb % v == 0 && q.x_sn % v == 0 &&
         q.o_sb % v == 0 && q.o_sn % v == 0;
}

// ---------------------------------------------------------------------------
// workspace layout of saf_tome_match
struct MatchLayout {
  size_t off_a, off_b, off_na, off_nb, off_rinv, off_ci, off_cv, off_nmax, off_nidx;
  size_t off_keys_out, off_vals_in, off_vals_out, off_dkey, off_dkey_out, off_dval_out, off_seg1,
      off_seg2, off_cub, cub_bytes, total;
};

size_t up256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

MatchLayout match_layout(int64_t B, int64_t Ns, int64_t Nd, int64_t Cp, int64_t r) {
  MatchLayout l{};
  size_t o = 0;
  auto take = [&](size_t bytes) {
    const size_t at = o;
    o = up256(o + bytes);
    return at;
  };
  l.off_a = take(B * Ns * Cp * 2);
  l.off_b = take(B * Nd * Cp * 2);
  l.off_na = take(B * Ns * 8);
  l.off_nb = take(B * Nd * 8);
  l.off_rinv = take(B * ((Nd + 3) & ~3) * 4);
  l.off_ci = take(B * Ns * kCand * 4);
  l.off_cv = take(B * Ns * kCand * 4);
  l.off_nmax = take(B * Ns * 8);
  l.off_nidx = take(B * Ns * 4);
  l.off_keys_out = take(B * Ns * 8);
  l.off_vals_in = take(B * Ns * 4);
  l.off_vals_out = take(B * Ns * 4);
  l.off_dkey = take(B * (r > 0 ? r : 1) * 4);
  l.off_dkey_out = take(B * (r > 0 ? r : 1) * 4);
  l.off_dval_out = take(B * (r > 0 ? r : 1) * 4);
  l.off_seg1 = take((B + 1) * 4);
  l.off_seg2 = take((B + 1) * 4);
  // CUB temp storage: the larger of the two segmented sorts
  size_t t1 = 0, t2 = 0;
  cub::DeviceSegmentedRadixSort::SortPairsDescending(
      nullptr, t1, static_cast<const double*>(nullptr), static_cast<double*>(nullptr),
      static_cast<const int*>(nullptr), static_cast<int*>(nullptr), static_cast<int>(B * Ns),
      static_cast<int>(B), static_cast<const int*>(nullptr), static_cast<const int*>(nullptr));
  cub::DeviceSegmentedRadixSort::SortPairs(
      nullptr, t2, static_cast<const int*>(nullptr), static_cast<int*>(nullptr),
      static_cast<const int*>(nullptr), static_cast<int*>(nullptr),
      static_cast<int>(B * (r > 0 ? r : 1)), static_cast<int>(B), static_cast<const int*>(nullptr),
      static_cast<const int*>(nullptr));
  l.cub_bytes = t1 > t2 ? t1 : t2;
  l.off_cub = take(l.cub_bytes);
  l.total = o;
  return l;
}

int64_t pad_c(int64_t C) { return (C + kTK - 1) / kTK * kTK; }

int32_t make_rows_map(CUtensorMap* map, void* base, int64_t B, int64_t rows, int64_t Cp, int box_rows,
                      bool bf16) {
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(Cp), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(Cp) * 2, static_cast<cuuint64_t>(rows * Cp) * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(kTK), static_cast<cuuint32_t>(box_rows), 1u};
  const CUresult r = encode_tensor_map(
      map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, base, dims,
      strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
  return r == CUDA_SUCCESS ? SAF_OK : SAF_ERR_STRIDE;
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" size_t saf_tome_match_workspace_bytes(int64_t B, int64_t Ns, int64_t Nd, int64_t C,
                                                 int32_t r) {
  if (B <= 0 || Ns <= 0 || Nd <= 0 || C <= 0) return 0;
  return match_layout(B, Ns, Nd, pad_c(C), r < 0 ? 0 : (r > Ns ? Ns : r)).total;
}

extern "C" int32_t saf_tome_match(const void* metric, int32_t dtype, int64_t B, int64_t N,
                                  int64_t C, int64_t stride_b, int64_t stride_n,
                                  const int32_t* a_idx, int64_t Ns, const int32_t* b_idx,
                                  int64_t Nd, int32_t r, const saf_tome_plan* plan,
                                  void* workspace, size_t workspace_bytes, void* stream) {
  if (metric == nullptr || a_idx == nullptr || b_idx == nullptr || plan == nullptr) return SAF_ERR_ARG;
  if (dtype != SAF_BF16 && dtype != SAF_F16) return SAF_ERR_DTYPE;
  if (B <= 0 || N <= 0 || C <= 0 || Ns <= 0 || Nd <= 0 || Ns + Nd > N) return SAF_ERR_SHAPE;
  if (B > 65535 || N >= (int64_t(1) << 30) || C > 65536) return SAF_ERR_SHAPE;
  if (stride_n < C || stride_b < 0) return SAF_ERR_STRIDE;
  if (r < 0) return SAF_ERR_ARG;
  const int64_t rr = r > Ns ? Ns : r;  // "can't reduce more than the # tokens in src"
  if (rr > 0 && (plan->src_idx == nullptr || plan->dst_idx == nullptr)) return SAF_ERR_ARG;
  if (rr < Ns && plan->unm_idx == nullptr) return SAF_ERR_ARG;
  if (plan->counter == nullptr || plan->dst_ptr == nullptr || plan->dst_src == nullptr)
    return SAF_ERR_ARG;
  const int64_t Cp = pad_c(C);
  const MatchLayout lay = match_layout(B, Ns, Nd, Cp, rr);
  if (workspace == nullptr || workspace_bytes < lay.total ||
      (reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return SAF_ERR_WORKSPACE;
  DeviceScope dev_scope;
  int32_t rc = dev_scope.bind(metric);
  if (rc != SAF_OK) return rc;
  if (!current_device_is_sm100()) return SAF_ERR_UNSUPPORTED;
  unsigned int* status = device_status_ptr();
  if (status == nullptr) return SAF_ERR_CUDA;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* A = ws + lay.off_a;
  void* Bm = ws + lay.off_b;
  double* na = reinterpret_cast<double*>(ws + lay.off_na);
  double* nb = reinterpret_cast<double*>(ws + lay.off_nb);
  float* rinv = reinterpret_cast<float*>(ws + lay.off_rinv);
  int32_t* ci = reinterpret_cast<int32_t*>(ws + lay.off_ci);
  float* cv = reinterpret_cast<float*>(ws + lay.off_cv);
  double* nmax = plan->node_max ? plan->node_max : reinterpret_cast<double*>(ws + lay.off_nmax);
  int32_t* nidx = plan->node_idx ? plan->node_idx : reinterpret_cast<int32_t*>(ws + lay.off_nidx);
  const bool bf16 = dtype == SAF_BF16;

  // 1. gather src / dst rows (zero-padded to Cp) and their exact norms
  GatherParams g{metric, stride_b, stride_n, static_cast<int>(B), static_cast<int>(N),
                 static_cast<int>(C), static_cast<int>(Cp), a_idx, static_cast<int>(Ns), A, na,
                 nullptr, status};
  dim3 gg_a(static_cast<unsigned>((Ns + 8 * kGatherRows - 1) / (8 * kGatherRows)), static_cast<unsigned>(B));
  GatherParams gb = g;
  gb.idx = b_idx;
  gb.n_rows = static_cast<int>(Nd);
  gb.out = Bm;
  gb.sqnorm = nb;
  gb.rinv = rinv;
  dim3 gg_b(static_cast<unsigned>((Nd + 8 * kGatherRows - 1) / (8 * kGatherRows)), static_cast<unsigned>(B));
  if (bf16) {
    tome_gather_kernel<__nv_bfloat16><<<gg_a, 256, 0, st>>>(g);
    tome_gather_kernel<__nv_bfloat16><<<gg_b, 256, 0, st>>>(gb);
  } else {
    tome_gather_kernel<__half><<<gg_a, 256, 0, st>>>(g);
    tome_gather_kernel<__half><<<gg_b, 256, 0, st>>>(gb);
  }
  SAF_CUDA_TRY(cudaGetLastError());

  // 2. tensor-core scores with the top-8 epilogue
  CUtensorMap ma, mb;
  if ((rc = make_rows_map(&ma, A, B, Ns, Cp, kTM, bf16)) != SAF_OK) return rc;
  if ((rc = make_rows_map(&mb, Bm, B, Nd, Cp, kTN, bf16)) != SAF_OK) return rc;
  ScoreParams sp{static_cast<int>(B), static_cast<int>(Ns), static_cast<int>(Nd), static_cast<int>(Cp),
                 na, rinv, ci, cv, status, wait_budget_ns()};
  // persistent: one CTA per SM over the (128-row block, batch row) items
  int score_dev = 0, score_sms = 0;
  SAF_CUDA_TRY(cudaGetDevice(&score_dev));
  SAF_CUDA_TRY(cudaDeviceGetAttribute(&score_sms, cudaDevAttrMultiProcessorCount, score_dev));
  const int64_t score_items = ((Ns + kTM - 1) / kTM) * B;
  const dim3 sg(static_cast<unsigned>(std::min<int64_t>(score_items, score_sms)));
  // narrow metrics (per-head [k, |k|, v, |v|]) keep A resident; wide ones stream it
  const bool res = Cp / kTK <= kResChunks;
  auto launch = [&](auto kern, int smem) -> cudaError_t {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    kern<<<sg, kScoreThreads, smem, st>>>(ma, mb, sp);
    return cudaGetLastError();
  };
  if (bf16)
    SAF_CUDA_TRY(res ? launch(tome_score_kernel<true, true>, ScoreLayoutT<true>::kDynSmem)
                     : launch(tome_score_kernel<true, false>, ScoreLayoutT<false>::kDynSmem));
  else
    SAF_CUDA_TRY(res ? launch(tome_score_kernel<false, true>, ScoreLayoutT<true>::kDynSmem)
                     : launch(tome_score_kernel<false, false>, ScoreLayoutT<false>::kDynSmem));

  // 3. exact fp64 re-score of the candidates
  ExactParams ep{A, Bm, na, nb, ci, cv, static_cast<int>(B), static_cast<int>(Ns), static_cast<int>(Nd),
                 static_cast<int>(Cp), nmax, nidx};
  const bool exact_short = Cp <= 32 * kExactCols;
  const dim3 eg(static_cast<unsigned>((Ns + 7) / 8), static_cast<unsigned>(B));
  if (bf16) {
    if (exact_short) tome_exact_kernel<__nv_bfloat16, true><<<eg, 256, 0, st>>>(ep);
    else tome_exact_kernel<__nv_bfloat16, false><<<eg, 256, 0, st>>>(ep);
  } else {
    if (exact_short) tome_exact_kernel<__half, true><<<eg, 256, 0, st>>>(ep);
    else tome_exact_kernel<__half, false><<<eg, 256, 0, st>>>(ep);
  }
  SAF_CUDA_TRY(cudaGetLastError());

  // 4. stable sort of node_max (descending) per batch row
  int* seg1 = reinterpret_cast<int*>(ws + lay.off_seg1);
  int* seg2 = reinterpret_cast<int*>(ws + lay.off_seg2);
  int32_t* vals_in = reinterpret_cast<int32_t*>(ws + lay.off_vals_in);
  int32_t* order = reinterpret_cast<int32_t*>(ws + lay.off_vals_out);
  double* keys_out = reinterpret_cast<double*>(ws + lay.off_keys_out);
  tome_offsets_kernel<<<static_cast<unsigned>((B + 256) / 256), 256, 0, st>>>(static_cast<int>(B), static_cast<int>(Ns), seg1);
  tome_iota_kernel<<<dim3(static_cast<unsigned>((Ns + 255) / 256), static_cast<unsigned>(B)), 256, 0, st>>>(
      static_cast<int>(B), static_cast<int>(Ns), vals_in);
  if (Ns <= kSortCap) {
    SAF_CUDA_TRY((block_sort<double, true>(nmax, nullptr, nullptr, order, static_cast<int>(B), static_cast<int>(Ns), 64, st)));
  } else {
    size_t tb = lay.cub_bytes;
    SAF_CUDA_TRY(cub::DeviceSegmentedRadixSort::SortPairsDescending(
        ws + lay.off_cub, tb, nmax, keys_out, vals_in, order, static_cast<int>(B * Ns),
        static_cast<int>(B), seg1, seg1 + 1, 0, 64, st));
  }

  // 5. plan: src / dst / unm indices, token map, dst -> src lists, counters
  int32_t* dkey = reinterpret_cast<int32_t*>(ws + lay.off_dkey);
  int32_t* dkey_out = reinterpret_cast<int32_t*>(ws + lay.off_dkey_out);
  FinalParams fp{static_cast<int>(B), static_cast<int>(Ns), static_cast<int>(Nd), static_cast<int>(N),
                 static_cast<int>(rr), order, nidx, a_idx, b_idx, plan->unm_idx, plan->src_idx,
                 plan->dst_idx, dkey, reinterpret_cast<int32_t*>(ws + lay.off_dval_out), plan->token_map};
  const int64_t nmax_k = Ns > Nd ? Ns : Nd;
  tome_final_kernel<<<dim3(static_cast<unsigned>((nmax_k + 255) / 256), static_cast<unsigned>(B)), 256, 0, st>>>(fp);
  SAF_CUDA_TRY(cudaGetLastError());
  if (rr > 0) {
    tome_offsets_kernel<<<static_cast<unsigned>((B + 256) / 256), 256, 0, st>>>(static_cast<int>(B), static_cast<int>(rr), seg2);
    int dst_bits = 1;  // dst keys lie in [0, Nd)
    while ((int64_t(1) << dst_bits) < Nd) ++dst_bits;
    if (rr <= kSortCap) {
      SAF_CUDA_TRY((block_sort<int32_t, false>(dkey, reinterpret_cast<int32_t*>(ws + lay.off_dval_out),
                                               dkey_out, plan->dst_src, static_cast<int>(B), static_cast<int>(rr),
                                               dst_bits, st)));
    } else {
      size_t tb2 = lay.cub_bytes;
      SAF_CUDA_TRY(cub::DeviceSegmentedRadixSort::SortPairs(
          ws + lay.off_cub, tb2, dkey, dkey_out, reinterpret_cast<int32_t*>(ws + lay.off_dval_out),
          plan->dst_src, static_cast<int>(B * rr), static_cast<int>(B), seg2, seg2 + 1, 0, dst_bits, st));
    }
  }
  tome_dstptr_kernel<<<dim3(static_cast<unsigned>((Nd + 1 + 255) / 256), static_cast<unsigned>(B)), 256, 0, st>>>(
      static_cast<int>(B), static_cast<int>(Nd), static_cast<int>(rr), dkey_out, plan->dst_ptr,
      plan->counter, plan->log_count);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

namespace {
int32_t check_rows(const void* p, int32_t dtype) {
  if (p == nullptr) return SAF_ERR_ARG;
  if (dtype != SAF_BF16 && dtype != SAF_F16 && dtype != SAF_F32) return SAF_ERR_DTYPE;
  return SAF_OK;
}
}  // namespace

// ---------------------------------------------------------------------------
// MergeAttention's matching metric [k, |k|, v, |v|] of the video tokens.
// One warp per token row: lane l holds the 16-bit pairs at words l, l + 32
// of the row (coalesced 4-byte loads), squares them in fp64 and adds
// (x[2w]^2 + x[2w+1]^2) for its words in ascending order; the lanes' sums are
// combined by the xor butterfly 16, 8, 4, 2, 1; the fp64 sqrt is rounded
// once to the 16-bit type.
namespace saf {
namespace {
constexpr int kKvMaxD = 128;
constexpr int kKvRowsPerWarp = 4;

struct KvMetricParams {
  const void* k;
  const void* v;
  void* out;  // [B*H, S - text, 2D + 2]
  int64_t k_sb, k_sh, k_ss, v_sb, v_sh, v_ss;
  int H, S, D, text;
};

template <typename T>
__global__ void __launch_bounds__(256) tome_kv_metric_kernel(const KvMetricParams p) {
  const int N = p.S - p.text;
  const int g = blockIdx.y, b = g / p.H, h = g % p.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int W = p.D / 2, C = 2 * p.D + 2;
  const int n_first = (blockIdx.x * 8 + warp) * kKvRowsPerWarp;
  const T* kb = static_cast<const T*>(p.k) + b * p.k_sb + h * p.k_sh;
  const T* vb = static_cast<const T*>(p.v) + b * p.v_sb + h * p.v_sh;
  uint32_t w[kKvRowsPerWarp][2][2];
#pragma unroll
  for (int r = 0; r < kKvRowsPerWarp; ++r) {
    const int n = n_first + r;
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      const T* x = (part == 0 ? kb : vb) + static_cast<int64_t>(p.text + n) * (part == 0 ? p.k_ss : p.v_ss);
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int word = lane + 32 * i;
        w[r][part][i] = (n < N && word < W) ? __ldg(reinterpret_cast<const uint32_t*>(x) + word) : 0u;
      }
    }
  }
#pragma unroll
  for (int r = 0; r < kKvRowsPerWarp; ++r) {
    const int n = n_first + r;
    if (n >= N) break;
    T* o = static_cast<T*>(p.out) + (static_cast<int64_t>(g) * N + n) * C;
    uint32_t nrm_bits[2];
#pragma unroll
    for (int part = 0; part < 2; ++part) {
      double acc = 0.0;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int word = lane + 32 * i;
        if (word < W) {
          const T* e = reinterpret_cast<const T*>(&w[r][part][i]);
          const double a = static_cast<double>(to_f(e[0])), c = static_cast<double>(to_f(e[1]));
          acc = __dadd_rn(acc, __dadd_rn(__dmul_rn(a, a), __dmul_rn(c, c)));
        }
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) acc = __dadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, m));
      const double nrm = sqrt(acc);
      if constexpr (std::is_same<T, __nv_bfloat16>::value) nrm_bits[part] = __bfloat16_as_ushort(__double2bfloat16(nrm));
      else nrm_bits[part] = __half_as_ushort(__double2half(nrm));
    }
    // The row [k (D), |k|, v (D), |v|] as 4-byte words (rows are 4-byte
    // aligned, C = 2D + 2 is even): words [0, W) are k as loaded, word W is
    // (|k|, v0), words W + 1 + i are (v[2i+1], v[2i+2]) -- v shifted by one
    // 16-bit place, taken from this lane's word and the next one -- and word
    // 2W is (v[D-1], |v|).
    uint32_t* o32 = reinterpret_cast<uint32_t*>(o);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int word = lane + 32 * i;
      if (word < W) o32[word] = w[r][0][i];
      const uint32_t cur = w[r][1][i];
      uint32_t nxt = __shfl_down_sync(0xffffffffu, cur, 1);
      const uint32_t wrap = __shfl_sync(0xffffffffu, w[r][1][i + 1 < 2 ? i + 1 : i], 0);
      if (lane == 31) nxt = wrap;
      if (word < W - 1) o32[W + 1 + word] = (cur >> 16) | (nxt << 16);
      if (word == W - 1) o32[2 * W] = (cur >> 16) | (nrm_bits[1] << 16);
    }
    if (lane == 0) o32[W] = nrm_bits[0] | (w[r][1][0] << 16);
  }
}
}  // namespace
}  // namespace saf

extern "C" int32_t saf_tome_kv_metric(const saf_tensor4* k, const saf_tensor4* v, int32_t text_len,
                                      void* out, void* stream) {
  if (k == nullptr || v == nullptr || out == nullptr) return SAF_ERR_ARG;
  int32_t rc;
  if ((rc = check_tensor4(k)) != SAF_OK || (rc = check_tensor4(v)) != SAF_OK) return rc;
  if (k->dtype != v->dtype) return SAF_ERR_DTYPE;
  if (k->dtype != SAF_BF16 && k->dtype != SAF_F16) return SAF_ERR_DTYPE;
  if (k->B != v->B || k->H != v->H || k->S != v->S || k->D != v->D) return SAF_ERR_SHAPE;
  if (text_len < 0 || text_len >= k->S || k->B * k->H > 65535) return SAF_ERR_SHAPE;
  if (k->D % 2 != 0 || k->D > kKvMaxD) return SAF_ERR_UNSUPPORTED;
  const saf_tensor4* kv[2] = {k, v};
  for (const saf_tensor4* x : kv)  // 4-byte aligned rows for the staged loads
    if ((reinterpret_cast<uintptr_t>(x->data) & 3) != 0 || x->stride_s % 2 || x->stride_h % 2 ||
        x->stride_b % 2)
      return SAF_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(out) & 3) != 0) return SAF_ERR_STRIDE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(k->data)) != SAF_OK) return rc;
  KvMetricParams p{k->data, v->data, out, k->stride_b, k->stride_h, k->stride_s, v->stride_b,
                   v->stride_h, v->stride_s, static_cast<int>(k->H), static_cast<int>(k->S),
                   static_cast<int>(k->D), text_len};
  const int N = static_cast<int>(k->S) - text_len;
  const int per_cta = 8 * kKvRowsPerWarp;
  dim3 grid(static_cast<unsigned>((N + per_cta - 1) / per_cta), static_cast<unsigned>(k->B * k->H));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (k->dtype == SAF_BF16) tome_kv_metric_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(p);
  else tome_kv_metric_kernel<__half><<<grid, 256, 0, st>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

extern "C" int32_t saf_tome_merge(const void* x, void* out, int32_t dtype, int64_t B, int64_t C,
                                  int64_t x_stride_b, int64_t x_stride_n, int64_t o_stride_b,
                                  int64_t o_stride_n, int32_t text_len, const int32_t* a_idx,
                                  int64_t Ns, const int32_t* b_idx, int64_t Nd, int32_t r,
                                  const saf_tome_plan* plan, void* stream) {
  int32_t rc;
  if ((rc = check_rows(x, dtype)) != SAF_OK || (rc = check_rows(out, dtype)) != SAF_OK) return rc;
  if (plan == nullptr || a_idx == nullptr || b_idx == nullptr || plan->counter == nullptr ||
      plan->dst_ptr == nullptr || plan->dst_src == nullptr)
    return SAF_ERR_ARG;
  if (B <= 0 || C <= 0 || Ns <= 0 || Nd <= 0 || text_len < 0 || r < 0 || r > Ns || B > 65535)
    return SAF_ERR_SHAPE;
  if (r < Ns && plan->unm_idx == nullptr) return SAF_ERR_ARG;
  if (x_stride_n < C || o_stride_n < C) return SAF_ERR_STRIDE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(x)) != SAF_OK) return rc;
  RowCopyParams q{x, out, x_stride_b, x_stride_n, o_stride_b, o_stride_n, static_cast<int>(B),
                  static_cast<int>(C), text_len, static_cast<int>(Ns), static_cast<int>(Nd), r, 0,
                  a_idx, b_idx, plan->unm_idx, plan->counter, plan->dst_ptr, plan->dst_src, nullptr};
  const int64_t rows = text_len + (Ns - r) + Nd;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t elem = dtype == SAF_F32 ? 4 : 2;
  if (rows_vec16(q, elem)) {
    const int chunks = static_cast<int>(C * static_cast<int64_t>(elem) / 16);
    const int64_t total = rows * chunks;
    dim3 vgrid(static_cast<unsigned>((total + 255) / 256), static_cast<unsigned>(B));
    switch (dtype) {
      case SAF_BF16: tome_merge_vec_kernel<__nv_bfloat16><<<vgrid, 256, 0, st>>>(q, chunks, total); break;
      case SAF_F16: tome_merge_vec_kernel<__half><<<vgrid, 256, 0, st>>>(q, chunks, total); break;
      default: tome_merge_vec_kernel<float><<<vgrid, 256, 0, st>>>(q, chunks, total); break;
    }
    SAF_CUDA_TRY(cudaGetLastError());
    return SAF_OK;
  }
  dim3 grid(static_cast<unsigned>((rows + 7) / 8), static_cast<unsigned>(B));
  switch (dtype) {
    case SAF_BF16: tome_merge_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(q); break;
    case SAF_F16: tome_merge_kernel<__half><<<grid, 256, 0, st>>>(q); break;
    default: tome_merge_kernel<float><<<grid, 256, 0, st>>>(q); break;
  }
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

extern "C" int32_t saf_tome_unmerge(const void* y, void* out, int32_t dtype, int64_t B, int64_t C,
                                    int64_t y_stride_b, int64_t y_stride_n, int64_t o_stride_b,
                                    int64_t o_stride_n, int32_t text_len, int64_t N,
                                    const int32_t* token_map, void* stream) {
  int32_t rc;
  if ((rc = check_rows(y, dtype)) != SAF_OK || (rc = check_rows(out, dtype)) != SAF_OK) return rc;
  if (token_map == nullptr) return SAF_ERR_ARG;
  if (B <= 0 || C <= 0 || N <= 0 || text_len < 0 || B > 65535) return SAF_ERR_SHAPE;
  if (y_stride_n < C || o_stride_n < C) return SAF_ERR_STRIDE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(y)) != SAF_OK) return rc;
  RowCopyParams q{y, out, y_stride_b, y_stride_n, o_stride_b, o_stride_n, static_cast<int>(B),
                  static_cast<int>(C), text_len, 0, 0, 0, static_cast<int>(N), nullptr, nullptr,
                  nullptr, nullptr, nullptr, nullptr, token_map};
  const int64_t rows = text_len + N;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t elem = dtype == SAF_F32 ? 4 : 2;
  if (rows_vec16(q, elem)) {
    const int chunks = static_cast<int>(C * static_cast<int64_t>(elem) / 16);
    const int64_t total = rows * chunks;
    dim3 vgrid(static_cast<unsigned>((total + 255) / 256), static_cast<unsigned>(B));
    switch (dtype) {
      case SAF_BF16: tome_unmerge_vec_kernel<__nv_bfloat16><<<vgrid, 256, 0, st>>>(q, chunks, total); break;
      case SAF_F16: tome_unmerge_vec_kernel<__half><<<vgrid, 256, 0, st>>>(q, chunks, total); break;
      default: tome_unmerge_vec_kernel<float><<<vgrid, 256, 0, st>>>(q, chunks, total); break;
    }
    SAF_CUDA_TRY(cudaGetLastError());
    return SAF_OK;
  }
  dim3 grid(static_cast<unsigned>((rows + 7) / 8), static_cast<unsigned>(B));
  switch (dtype) {
    case SAF_BF16: tome_unmerge_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(q); break;
    case SAF_F16: tome_unmerge_kernel<__half><<<grid, 256, 0, st>>>(q); break;
    default: tome_unmerge_kernel<float><<<grid, 256, 0, st>>>(q); break;
  }
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
