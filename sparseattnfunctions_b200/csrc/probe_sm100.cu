// probe_sm100.cu -- probe mass of sampled query rows on tcgen05 (sm_100a).
//
// Follows probe_solver._probe_num of the reference's LocalGlobalAttention
// (special_attentions/LocalGlobalAttention.py:50-62): for R sampled query
// rows of every head and all Sk keys,
//   att  = softmax_keys( round16(q_r . k) * scale )        (16-bit tensor)
//   mass = round16( sum over heads and sampled rows of att )
// with the reference's 16-bit roundings reproduced: the product rounded to
// the input type (the matmul's output), scale = 1/sqrt(64) (exact), the
// softmax in fp32 over the rounded logits with its output rounded to the
// input type, the sum accumulated in fp32 and rounded once.  (The reference
// then masks and sorts; masked_topn in local_global.cu does that.)
//
// Two passes of one kernel, each "one A tile fixed, B tiles streaming":
//   pass 1 (row statistics)  A = 128 sampled rows, B = key tiles of one
//          chunk of the keys.  S = A B^T in TMEM, one softmax thread per
//          sampled row keeps the running max m and sum l over the chunk.
//   merge  per row: m = max over chunks, l = sum l_c exp(m_c - m); stores
//          (-m log2 e, 1/l) per row (rows past R: (0, 0)).
//   pass 2 (column sums)     A = 128 keys, B = the sampled-row tiles.
//          S^T = K Q^T in TMEM, one thread per key sums the rounded
//          probabilities over every sampled row; the rows' statistics come
//          with each B tile (1 KB bulk copy next to the TMA tile).
//   heads  mass[b, key] = round16(sum over h, ascending, of the pass-2 sums).
// Every sum has a fixed order, so the mass is the same on every run.
//
// Kernel layout (persistent, 2 CTAs per SM, 192 threads):
//   warp 0     TMA producer (A tile per work item, 3-stage B ring)
//   warp 1     TMEM allocator and single-thread tcgen05.mma issuer
//              (4 x K=16 MMAs per tile into one of two 128-column S buffers)
//   warps 2-5  one thread per TMEM lane (warp w reads lanes 32 (w % 4) ...)
// Every mbarrier wait has a time budget; on expiry the CTA raises its abort
// flag and the device status word, drains its copies and MMAs, frees TMEM
// and returns.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cmath>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kTile = 128;
constexpr int kD = 64;
constexpr int kBS = 3;              // B stages
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 256;  // two S buffers
constexpr uint32_t kTileBytes = kTile * kD * 2;
constexpr uint32_t kStatBytes = kTile * 8;  // (-m log2e, 1/l) per row
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kScale = 0.125f;  // 1 / sqrt(64)

struct ProbeParams {
  int pass;         // 1 or 2
  int G, H;         // heads (B * H), heads per batch
  int n_a;          // A tiles per head
  int n_b;          // B tiles per head
  int chunks;       // pass 1: key chunks
  int chunk_tiles;  // pass 1: B tiles per chunk
  int Sk, R, R_pad;
  int items;
  const float2* stats;  // pass 2: [G, R_pad] (-m log2e, 1/l)
  float* part_m;        // pass 1: [G, chunks, R_pad]
  float* part_l;
  float* part_mass;     // pass 2: [G, Sk]
  unsigned int* status;
  uint64_t budget_ns;
};

struct Smem {
  alignas(1024) uint8_t a[kTileBytes];
  alignas(1024) uint8_t b[kBS][kTileBytes];
  alignas(16) float2 stats[kBS][kTile];
  alignas(8) uint64_t bar_a_full, bar_a_empty, bar_drain;
  uint64_t bar_b_full[kBS], bar_b_empty[kBS];
  uint64_t bar_s_full[2], bar_s_empty[2];
  uint32_t tmem_base;
  int abort_flag;
};

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(bar)
      : "memory");
}

// Work item -> head, A tile, B tile range.
struct Item {
  int g, a, b0, b1;
};
__device__ __forceinline__ Item item_of(const ProbeParams& p, int it) {
  Item r;
  if (p.pass == 1) {
    const int c = it % p.chunks;
    const int t = it / p.chunks;
    r.a = t % p.n_a;
    r.g = t / p.n_a;
    r.b0 = c * p.chunk_tiles;
    r.b1 = min(p.n_b, r.b0 + p.chunk_tiles);
    r.b0 = min(r.b0, r.b1);
  } else {
    r.a = it % p.n_a;
    r.g = it / p.n_a;
    r.b0 = 0;
    r.b1 = p.n_b;
  }
  return r;
}

// 16-bit rounding of two fp32 values, back to fp32 (round to nearest even).
template <bool kBF16>
__device__ __forceinline__ void round16x2(float& lo, float& hi) {
  if constexpr (kBF16) {
    const uint32_t u = pack_bf16x2(lo, hi);
    lo = __uint_as_float(u << 16);
    hi = __uint_as_float(u & 0xffff0000u);
  } else {
    const uint32_t u = pack_f16x2(lo, hi);
    __half2 h2 = *reinterpret_cast<const __half2*>(&u);
    const float2 f = __half22float2(h2);
    lo = f.x;
    hi = f.y;
  }
}

template <bool kBF16>
__global__ void __launch_bounds__(kThreads, 2)
    probe_sm100_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b,
                       const ProbeParams p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &sm.abort_flag;
  const uint32_t sA = smem_u32(sm.a);
  auto sB = [&](int s) { return smem_u32(sm.b[s]); };
  const uint32_t bar_a_full = smem_u32(&sm.bar_a_full), bar_a_empty = smem_u32(&sm.bar_a_empty);
  auto bar_b_full = [&](int s) { return smem_u32(&sm.bar_b_full[s]); };
  auto bar_b_empty = [&](int s) { return smem_u32(&sm.bar_b_empty[s]); };
  auto bar_s_full = [&](int s) { return smem_u32(&sm.bar_s_full[s]); };
  auto bar_s_empty = [&](int s) { return smem_u32(&sm.bar_s_empty[s]); };
  const bool pass2 = p.pass == 2;

  if (threadIdx.x == 0) {
    sm.abort_flag = 0;
    mbar_init(bar_a_full, 1);
    mbar_init(bar_a_empty, 1);
    mbar_init(smem_u32(&sm.bar_drain), 1);
    for (int s = 0; s < kBS; ++s) {
      mbar_init(bar_b_full(s), 1);
      // pass 2: the softmax warps read the stage's row statistics too
      mbar_init(bar_b_empty(s), pass2 ? 5 : 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_s_full(s), 1);
      mbar_init(bar_s_empty(s), 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    int na = 0, nb = 0;
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      for (int it = blockIdx.x; it < p.items; it += gridDim.x) {
        const Item w = item_of(p, it);
        const int b = w.g / p.H, h = w.g % p.H;
        if (na > 0 && !mbar_wait(bar_a_empty, (na - 1) & 1, abort_flag, p.status, p.budget_ns)) break;
        mbar_arrive_expect_tx(bar_a_full, kTileBytes);
        tma_load_4d(sA, &tm_a, bar_a_full, 0, w.a * kTile, h, b);
        ++na;
        bool ok = true;
        for (int t = w.b0; t < w.b1; ++t) {
          const int s = nb % kBS;
          if (!mbar_wait(bar_b_empty(s), ((nb / kBS) & 1) ^ 1, abort_flag, p.status, p.budget_ns)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(bar_b_full(s), kTileBytes + (pass2 ? kStatBytes : 0u));
          tma_load_4d(sB(s), &tm_b, bar_b_full(s), 0, t * kTile, h, b);
          if (pass2)
            bulk_load(smem_u32(sm.stats[s]), p.stats + static_cast<int64_t>(w.g) * p.R_pad + t * kTile,
                      kStatBytes, bar_b_full(s));
          ++nb;
        }
        if (!ok) break;
      }
      // drain: the last load into A and into every B stage
      if (na > 0) mbar_drain(bar_a_full, (na - 1) & 1, p.status);
      for (int s = 0; s < kBS && s < nb; ++s) {
        const int last = s + ((nb - 1 - s) / kBS) * kBS;
        mbar_drain(bar_b_full(s), (last / kBS) & 1, p.status);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_f16(kTile, kTile, kBF16, false, false);
      int na = 0, nb = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
        const Item w = item_of(p, it);
        if (!mbar_wait(bar_a_full, na & 1, abort_flag, p.status, p.budget_ns)) break;
        ++na;
        for (int t = w.b0; t < w.b1; ++t) {
          const int s = nb % kBS, buf = nb & 1;
          if (!mbar_wait(bar_b_full(s), (nb / kBS) & 1, abort_flag, p.status, p.budget_ns) ||
              !mbar_wait(bar_s_empty(buf), ((nb >> 1) & 1) ^ 1, abort_flag, p.status, p.budget_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(sA + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(sB(s) + kk * 32, 16, 1024);
            tc_mma_ss(tmem + buf * kTile, ad, bd, kIdesc, kk > 0 ? 1u : 0u);
          }
          tc_commit(bar_s_full(buf));
          tc_commit(bar_b_empty(s));
          ++nb;
        }
        tc_commit(bar_a_empty);
      }
      const uint32_t bar_drain = smem_u32(&sm.bar_drain);
      tc_commit(bar_drain);
      mbar_drain(bar_drain, 0, p.status);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ softmax
    const int quarter = warp & 3;
    const int lrow = quarter * 32 + lane;  // TMEM lane = A row of the tile
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const float c1 = kScale * kLog2e;
    int nb = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < p.items && ok; it += gridDim.x) {
      const Item w = item_of(p, it);
      float m = -INFINITY, l = 0.f;  // pass 1, natural units of the scaled logits
      float acc0 = 0.f, acc1 = 0.f;  // pass 2
      for (int t = w.b0; t < w.b1; ++t) {
        const int s = nb % kBS, buf = nb & 1;
        if (!mbar_wait(bar_s_full(buf), (nb >> 1) & 1, abort_flag, p.status, p.budget_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t r[128];
        {
          uint32_t (&r0)[64] = *reinterpret_cast<uint32_t(*)[64]>(&r[0]);
          uint32_t (&r1)[64] = *reinterpret_cast<uint32_t(*)[64]>(&r[64]);
          const uint32_t ta = tmem + lane_addr + buf * kTile;
          tmem_ld64(ta, r0);
          tmem_ld64(ta + 64, r1);
          tmem_wait_ld(r0);
          tmem_wait_ld(r1);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(bar_s_empty(buf));
        if (!pass2) {
          // keys of this B tile past Sk are masked
          const int nv = min(kTile, p.Sk - t * kTile);
          float mx = -INFINITY;
#pragma unroll
          for (int c = 0; c < kTile; c += 2) {
            float lo = __uint_as_float(r[c]), hi = __uint_as_float(r[c + 1]);
            round16x2<kBF16>(lo, hi);
            if (c >= nv) lo = -INFINITY;
            if (c + 1 >= nv) hi = -INFINITY;
            r[c] = __float_as_uint(lo);
            r[c + 1] = __float_as_uint(hi);
            mx = fmax3(mx, lo, hi);
          }
          const float mn = fmaxf(m, mx * kScale);
          const float nml = -mn * kLog2e;
          const f2 cc = mk2(c1, c1), nn = mk2(nml, nml);
          f2 sum = mk2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < kTile; c += 2) {
            const f2 x = fma2(mk2(__uint_as_float(r[c]), __uint_as_float(r[c + 1])), cc, nn);
            sum = add2(sum, mk2(ex2_approx(lo2(x)), ex2_approx(hi2(x))));
          }
          l = (m == -INFINITY ? 0.f : l * ex2_approx((m - mn) * kLog2e)) + lo2(sum) + hi2(sum);
          m = mn;
        } else {
          // B tile rows' statistics, staged with the tile (visible once its
          // barrier phase completed; the MMA issuer waited on it already)
          if (!mbar_wait(bar_b_full(s), (nb / kBS) & 1, abort_flag, p.status, p.budget_ns)) {
            ok = false;
            break;
          }
          const float4* st = reinterpret_cast<const float4*>(sm.stats[s]);
          const f2 cc = mk2(c1, c1);
          f2 acc = mk2(0.f, 0.f);
#pragma unroll
          for (int c = 0; c < kTile; c += 2) {
            const float4 sv = st[c >> 1];  // rows c, c+1: (-m log2e, 1/l) each
            float lo = __uint_as_float(r[c]), hi = __uint_as_float(r[c + 1]);
            round16x2<kBF16>(lo, hi);
            const f2 x = fma2(mk2(lo, hi), cc, mk2(sv.x, sv.z));
            f2 e = mul2(mk2(ex2_approx(lo2(x)), ex2_approx(hi2(x))), mk2(sv.y, sv.w));
            float pa = lo2(e), pb = hi2(e);
            round16x2<kBF16>(pa, pb);
            acc = add2(acc, mk2(pa, pb));
          }
          acc0 += lo2(acc);
          acc1 += hi2(acc);
          __syncwarp();
          if (lane == 0) mbar_arrive(bar_b_empty(s));
        }
        ++nb;
      }
      if (!ok) break;
      // item epilogue
      const int row = w.a * kTile + lrow;
      if (!pass2) {
        if (row < p.R_pad) {
          const int c = w.b0 / p.chunk_tiles;
          const int64_t o = (static_cast<int64_t>(w.g) * p.chunks + c) * p.R_pad + row;
          p.part_m[o] = m;
          p.part_l[o] = l;
        }
      } else if (row < p.Sk) {
        p.part_mass[static_cast<int64_t>(w.g) * p.Sk + row] = acc0 + acc1;
      }
    }
  }
  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Per (head, row): combine the chunks' (m, l).
__global__ void probe_merge_kernel(const float* __restrict__ part_m, const float* __restrict__ part_l,
                                   int G, int chunks, int R, int R_pad, float2* __restrict__ stats) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(G) * R_pad) return;
  const int g = static_cast<int>(i / R_pad), r = static_cast<int>(i % R_pad);
  if (r >= R) {
    stats[i] = make_float2(0.f, 0.f);
    return;
  }
  float m = -INFINITY;
  for (int c = 0; c < chunks; ++c) m = fmaxf(m, part_m[(static_cast<int64_t>(g) * chunks + c) * R_pad + r]);
  float l = 0.f;
  for (int c = 0; c < chunks; ++c) {
    const int64_t o = (static_cast<int64_t>(g) * chunks + c) * R_pad + r;
    l += part_l[o] * expf(part_m[o] - m);
  }
  stats[i] = make_float2(-m * kLog2e, 1.f / l);
}

// mass[b, key] = round16(sum over heads of the pass-2 sums), as fp64.
template <bool kBF16>
__global__ void probe_heads_kernel(const float* __restrict__ part, int B, int H, int Sk, double* __restrict__ mass) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= static_cast<int64_t>(B) * Sk) return;
  const int b = static_cast<int>(i / Sk), key = static_cast<int>(i % Sk);
  float s = 0.f;
  for (int h = 0; h < H; ++h) s += part[(static_cast<int64_t>(b) * H + h) * Sk + key];
  float hi = 0.f;
  round16x2<kBF16>(s, hi);
  mass[i] = static_cast<double>(s);
}

constexpr int kChunkTiles = 18;

struct ProbeWs {
  float* part_m;
  float* part_l;
  float2* stats;
  float* part_mass;
};

size_t probe_ws_layout(int64_t G, int64_t Sk, int64_t R, ProbeWs* ws, void* base) {
  const int64_t R_pad = (R + kTile - 1) / kTile * kTile;
  const int64_t n_b1 = (Sk + kTile - 1) / kTile;
  const int64_t chunks = (n_b1 + kChunkTiles - 1) / kChunkTiles;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off += (bytes + 255) & ~size_t(255);
    return o;
  };
  const size_t o_m = take(G * chunks * R_pad * 4), o_l = take(G * chunks * R_pad * 4);
  const size_t o_s = take(G * R_pad * 8), o_pm = take(G * Sk * 4);
  if (ws != nullptr) {
    uint8_t* b = static_cast<uint8_t*>(base);
    ws->part_m = reinterpret_cast<float*>(b + o_m);
    ws->part_l = reinterpret_cast<float*>(b + o_l);
    ws->stats = reinterpret_cast<float2*>(b + o_s);
    ws->part_mass = reinterpret_cast<float*>(b + o_pm);
  }
  return off;
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" size_t saf_probe_workspace_bytes(int64_t B, int64_t H, int64_t Sk, int32_t n_samp) {
  if (B <= 0 || H <= 0 || Sk <= 0 || n_samp <= 0) return 0;
  return probe_ws_layout(B * H, Sk, n_samp, nullptr, nullptr) + 256;
}

extern "C" int32_t saf_probe_mass(const saf_tensor4* qs, const saf_tensor4* k, void* workspace,
                                  size_t workspace_bytes, double* mass_out, void* stream) {
  int32_t rc = check_tensor4(qs);
  if (rc != SAF_OK) return rc;
  if ((rc = check_tensor4(k)) != SAF_OK) return rc;
  if (qs->dtype != k->dtype || qs->B != k->B || qs->H != k->H || qs->D != k->D) return SAF_ERR_SHAPE;
  if (qs->dtype == SAF_F32 || qs->D != kD) return SAF_ERR_UNSUPPORTED;
  if (mass_out == nullptr) return SAF_ERR_ARG;
  if (k->S > (1 << 30) || qs->S > (1 << 30) || qs->B * qs->H > (1 << 20)) return SAF_ERR_SHAPE;
  const int64_t G = qs->B * qs->H;
  const size_t need = saf_probe_workspace_bytes(qs->B, qs->H, k->S, static_cast<int32_t>(qs->S));
  if (workspace == nullptr || workspace_bytes < need) return SAF_ERR_WORKSPACE;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(qs->data)) != SAF_OK) return rc;
  if (!current_device_is_sm100()) return SAF_ERR_UNSUPPORTED;
  unsigned int* status = device_status_ptr();
  if (status == nullptr) return SAF_ERR_CUDA;
  ProbeWs ws;
  void* base = reinterpret_cast<void*>((reinterpret_cast<uintptr_t>(workspace) + 255) & ~uintptr_t(255));
  probe_ws_layout(G, k->S, qs->S, &ws, base);
  CUtensorMap m_q, m_k;
  if ((rc = make_qkv_map(&m_q, qs, kTile)) != SAF_OK) return rc;
  if ((rc = make_qkv_map(&m_k, k, kTile)) != SAF_OK) return rc;
  const bool bf16 = qs->dtype == SAF_BF16;
  const size_t smem = sizeof(Smem) + 1024;
  auto kern = bf16 ? probe_sm100_kernel<true> : probe_sm100_kernel<false>;
  SAF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
  int dev = 0, sms = 148;
  SAF_CUDA_TRY(cudaGetDevice(&dev));
  SAF_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  cudaStream_t st = static_cast<cudaStream_t>(stream);

  ProbeParams p{};
  p.G = static_cast<int>(G);
  p.H = static_cast<int>(qs->H);
  p.Sk = static_cast<int>(k->S);
  p.R = static_cast<int>(qs->S);
  p.R_pad = (p.R + kTile - 1) / kTile * kTile;
  p.chunk_tiles = kChunkTiles;
  p.status = status;
  p.budget_ns = wait_budget_ns();
  // pass 1: A = sampled rows, B = key tiles in chunks
  p.pass = 1;
  p.n_a = p.R_pad / kTile;
  p.n_b = (p.Sk + kTile - 1) / kTile;
  p.chunks = (p.n_b + kChunkTiles - 1) / kChunkTiles;
  p.items = p.G * p.n_a * p.chunks;
  p.part_m = ws.part_m;
  p.part_l = ws.part_l;
  const int chunks = p.chunks;
  kern<<<std::min(p.items, 2 * sms), kThreads, smem, st>>>(m_q, m_k, p);
  SAF_CUDA_TRY(cudaGetLastError());
  const int64_t n_st = G * p.R_pad;
  probe_merge_kernel<<<static_cast<unsigned>((n_st + 255) / 256), 256, 0, st>>>(ws.part_m, ws.part_l, p.G, chunks,
                                                                              p.R, p.R_pad, ws.stats);
  SAF_CUDA_TRY(cudaGetLastError());
  // pass 2: A = key tiles, B = sampled-row tiles with their statistics
  p.pass = 2;
  p.n_a = (p.Sk + kTile - 1) / kTile;
  p.n_b = p.R_pad / kTile;
  p.chunks = 1;
  p.items = p.G * p.n_a;
  p.stats = ws.stats;
  p.part_mass = ws.part_mass;
  kern<<<std::min(p.items, 2 * sms), kThreads, smem, st>>>(m_k, m_q, p);
  SAF_CUDA_TRY(cudaGetLastError());
  const int64_t n = qs->B * k->S;
  if (bf16)
    probe_heads_kernel<true><<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        ws.part_mass, static_cast<int>(qs->B), p.H, p.Sk, mass_out);
  else
    probe_heads_kernel<false><<<static_cast<unsigned>((n + 255) / 256), 256, 0, st>>>(
        ws.part_mass, static_cast<int>(qs->B), p.H, p.Sk, mass_out);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
