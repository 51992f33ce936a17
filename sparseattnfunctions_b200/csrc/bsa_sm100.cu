// bsa_sm100.cu -- block-sparse flash attention for sm_100a (B200).
//
// Computes, for every query row i of head g = b*H + h,
//   o_i = sum_{j in live kv blocks} softmax_j(sm_scale * q_i . k_j + bias_j) v_j
// where the live kv blocks of query block i / block_m come from a CSR list.
// Semantics follow the reference Triton kernel
// (special_attentions/utils/block_sparse_attn_kernel.py:52-209): online
// softmax, fp32 statistics and accumulation, P rounded to the input type
// before the PV product, keys past seqlen_k masked to -inf (:74-89), and
// a row with no live block divided by a zero row sum (:201-203).  Unlike the
// reference, which walks every mask bit of a row (:167-199), only the listed
// blocks are visited.
//
// Design (persistent: 2 CTAs per SM, each taking 128-row query tiles of any
// head from a launch-wide counter until none is left):
//   warp 0      TMA producer: fetches the next tile index and hands it to the
//               other roles through a 2-slot ring in shared memory, loads Q
//               once the previous tile's QK^T products are done, then K / V
//               tiles of each live block (3-stage K ring, 2-stage V ring,
//               128B swizzle) and, with a key bias, the block's 16-bit
//               bias / sm_scale column tile (2-stage ring, 32B swizzle).
//   warp 1      TMEM allocator and single-thread tcgen05.mma issuer:
//               S = Q K^T (SS form) into TMEM (+ ones x bias^T: one more
//               K = 16 MMA that adds the key bias), then O += P V (TS form, P
//               read from TMEM) for the previous block.
//   warps 2,3   idle (they complete warpgroup 0 for the register split).
//   warps 4..7  softmax: one thread per query row (TMEM lane) holds the
//               row's BN scores of a block, so the block maximum needs no
//               exchange; the scores are read once into registers (so the
//               next QK^T may start at once) and P (bf16/f16 pairs) is
//               written into TMEM.  P is computed speculatively with the
//               running max; the max only moves when it grows by more than
//               2^8 (lazy rescale: P <= 256, exact after the final 1/l), and
//               then P is recomputed and O rescaled in TMEM.  Each tile ends
//               with O read back, normalised and stored by these warps.
//               Optionally (attention with a pooled map) they also store each
//               row's block maxima and log2-sum-exp.  Inside a visited block
//               the keys past Sk are masked, and, by template mode, the keys
//               outside the row's two key intervals (frame bands) or outside
//               the frames the head's frame x frame mask gives the row's frame.
// TMEM columns: S [0,128) | O [128,192) | P [192,256).  Block phases of all
// rings run on a block counter that continues across a CTA's tiles.
//
// Every mbarrier wait has a time budget; on expiry the CTA raises a shared
// abort flag and the device status word, drains the copies and MMAs it has in
// flight, frees TMEM and returns.
#include <atomic>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kBM = 128;       // query rows per CTA
constexpr int kD = 64;         // head dim handled by this kernel
constexpr int kKS = 2;         // K stages (3 measured 0.8 % slower at config 2)
constexpr int kVS = 2;         // V stages
constexpr int kThreads = 256;  // 8 warps = 2 warpgroups
// Register split: launched at 128 per thread (2 CTAs x 256 threads per SM);
// warpgroup 0 (producer and MMA issuer with the persistent tile loop, 2 idle
// warps) drops to 56, the softmax warpgroup (one thread per query row) rises
// to 200: 128*56 + 128*200 = 32768 = 256*128.  (32 / 224 spilled in the
// control loop and measured 5 % slower.)
constexpr uint32_t kRegsCtl = 56, kRegsSoftmax = 200;
static_assert(128 * kRegsCtl + 128 * kRegsSoftmax <= kThreads * 128, "register split");
constexpr uint32_t kTmemCols = 256;
constexpr uint32_t kColS = 0, kColO = 128, kColP = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units
// a split partial row: O (64 fp32), m, l, padded to 16-byte multiples so
// every row starts 16-byte aligned for the vector stores and loads
constexpr int kSplitRow = kD + 4;
#ifndef SAF_OVERFLOW_GUARD
#define SAF_OVERFLOW_GUARD 1
#endif

struct BsaParams {
  int B, H, Sq, Sk;
  int nbq, nbk;    // mask rows / columns
  int bm;          // mask block rows: 64 or 128
  int64_t col_capacity;
  const int32_t* row_ptr;  // [B*H, nbq+1]
  const int32_t* col_idx;
  const float* kv_bias;    // nullable
  int64_t bias_stride;     // per head, elements
  float scale_log2;        // sm_scale * log2(e)
  float inv_scale;         // 1 / sm_scale
  void* o;
  int64_t o_sb, o_sh, o_ss;  // element strides
  unsigned int* status;
  uint64_t budget_ns;
  int lead_tiles;  // query tiles per head scheduled first
  // split key ranges of the lead tiles: each lead tile's block list is cut
  // into `splits` work items whose unnormalised partial results (O, m, l per
  // row) go to split_part; the last item of a row to finish merges them
  int splits;         // the most work items a lead tile may be split into (1: none)
  float* split_part;  // [B*H, lead_tiles, splits, 128, kSplitRow], 16-byte aligned rows
  int* split_cnt;     // [B*H, lead_tiles, 128], zero on entry
  // nullable [Sq] int4: the key columns of query row r are limited to
  // [x, y) U [z, w) (frame-band masks); shared by every head
  const int4* row_ranges;
  // frame-mask mode: [B*H, frames] words, bit f2 of word f1 set when video
  // queries of frame f1 may see the video keys of frame f2; text rows and
  // text keys are always visible
  const uint32_t* frame_bits;
  int text_len, frame_len, frames;
  // nullable pooled-map outputs (attention with pooling): per visited key
  // block the row's maximum logit in log2 units, [B*H, nbk, Sq], and the
  // row's log2-sum-exp, [B*H, Sq]
  float* pool_scratch;  // [grid][2][list_cap][128] block maxima of each CTA's last two tiles
  float* pool_out;      // [B*H, nbp, nbk], zeroed: per-row block maxima pooled by atomic max
  int pool_block, nbp;
  // persistent schedule: query tiles per head, heads, and this launch's
  // [next tile, CTAs done] counters (zero on entry; the last CTA resets them)
  int n_tiles, BH;
  unsigned int* tile_ctr;
  int list_cap;  // entries of a tile's block list in shared memory (nbk rounded up to 8)
  int dense;     // every key block live (no CSR)
  // key-list mode: the keys of attention batch b are rows key_list[b, :key_len)
  // of batch key_batch[b] of k / v ([B_src, H, key_src_len, D] contiguous),
  // fetched row by row with TMA gather4 loads
  const int32_t* key_list;
  const int32_t* key_batch;
  int key_len, key_src_len, key_src_batches;
};

// Builds the live key blocks of one 128-row query tile into a list in shared
// memory (uint16 entries: column | row mask << 14) and returns its length;
// the 32 lanes of the producer warp build it together, before the tile is
// handed to the other roles, which then read it from shared memory.  With
// `dense` set every key block is listed (no CSR is read).  With
// 64-row mask blocks the tile covers two mask rows: their column lists are
// merged through two bitmaps of the key blocks (ascending, a column listed by
// both rows once) and the row mask says which half is live (bit 0 = rows
// [0,64), bit 1 = rows [64,128)).  Out-of-range columns are skipped and set
// the bad-index flag.
__device__ int build_tile_list(const BsaParams& p, int g, int tile, uint16_t* lst, uint32_t* bits, int lane) {
  if (p.dense) {  // every key block, no CSR
    for (int j = lane; j < p.nbk; j += 32) lst[j] = static_cast<uint16_t>(j | (3 << 14));
    return p.nbk;
  }
  const int32_t* rp = p.row_ptr + static_cast<int64_t>(g) * (p.nbq + 1);
  auto clampi = [&](int32_t x) -> int32_t {
    return x < 0 ? 0 : (static_cast<int64_t>(x) > p.col_capacity ? static_cast<int32_t>(p.col_capacity) : x);
  };
  const bool two_rows = (p.bm == 64);
  const int r0 = two_rows ? 2 * tile : tile;
  const int p0 = clampi(rp[r0]), e0 = clampi(rp[r0 + 1]);
  const uint32_t below = (1u << lane) - 1u;
  int n = 0;
  if (!two_rows) {
    for (int base = p0; base < e0; base += 32) {
      const int i = base + lane;
      int c = -1;
      bool v = false;
      if (i < e0) {
        c = p.col_idx[i];
        v = c >= 0 && c < p.nbk;
        if (!v) atomicOr(p.status, SAF_DEV_BADINDEX);
      }
      const uint32_t m = __ballot_sync(0xffffffffu, v);
      if (v) lst[n + __popc(m & below)] = static_cast<uint16_t>(c | (3 << 14));
      n += __popc(m);
    }
    return n;
  }
  int p1 = 0, e1 = 0;
  if (r0 + 1 < p.nbq) {
    p1 = clampi(rp[r0 + 1]);
    e1 = clampi(rp[r0 + 2]);
  }
  const int words = (p.nbk + 31) >> 5;
  uint32_t* ba = bits;
  uint32_t* bb = bits + words;
  for (int w = lane; w < 2 * words; w += 32) bits[w] = 0u;
  __syncwarp();
  auto mark = [&](int s, int e, uint32_t* set) {
    for (int i = s + lane; i < e; i += 32) {
      const int c = p.col_idx[i];
      if (c >= 0 && c < p.nbk)
        atomicOr(set + (c >> 5), 1u << (c & 31));
      else
        atomicOr(p.status, SAF_DEV_BADINDEX);
    }
  };
  mark(p0, e0, ba);
  mark(p1, e1, bb);
  __syncwarp();
  for (int w0 = 0; w0 < words; w0 += 32) {
    const int w = w0 + lane;
    const uint32_t a = w < words ? ba[w] : 0u, b = w < words ? bb[w] : 0u;
    uint32_t u = a | b;
    const int cnt = __popc(u);
    int incl = cnt;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += y;
    }
    int pos = n + incl - cnt;
    while (u != 0u) {
      const int bit = __ffs(u) - 1;
      u &= u - 1u;
      const uint32_t rmask = ((a >> bit) & 1u) | (((b >> bit) & 1u) << 1);
      lst[pos++] = static_cast<uint16_t>((w * 32 + bit) | (rmask << 14));
    }
    n += __shfl_sync(0xffffffffu, incl, 31);
  }
  return n;
}

// exp2 on the FMA pipe (for part of the elements, to offload the MUFU):
// 2^x = 2^n * 2^f with n = rint(x) (from adding 1.5 * 2^23) and
// f = x - n in [-1/2, 1/2]; 2^f by a degree-3 polynomial whose coefficients
// minimise the maximum relative error on [-1/2, 1/2] (Remez exchange; max
// relative error 7.5e-5 in fp32 -- below bf16 and f16 rounding of P); 2^n
// inserted into the exponent field with one integer multiply-add.  x is
// clamped to -126 so masked (-inf) and vanishing scores give a tiny
// positive number instead of a wrapped exponent.
constexpr float kExp2C0 = 0.9999280571937561f;
constexpr float kExp2C1 = 0.6932609677314758f;
constexpr float kExp2C2 = 0.2426111251115799f;
constexpr float kExp2C3 = 0.0551716685295105f;
constexpr float kRoundShift = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ f2 exp2_poly2(f2 x) {
  x = mk2(fmaxf(lo2(x), -126.f), fmaxf(hi2(x), -126.f));
  const f2 t = add2(x, mk2(kRoundShift, kRoundShift));       // n in the low mantissa bits
  const f2 n = add2(t, mk2(-kRoundShift, -kRoundShift));     // rint(x)
  const f2 f = fma2(n, mk2(-1.f, -1.f), x);                  // x - n
  f2 q = fma2(mk2(kExp2C3, kExp2C3), f, mk2(kExp2C2, kExp2C2));
  q = fma2(q, f, mk2(kExp2C1, kExp2C1));
  q = fma2(q, f, mk2(kExp2C0, kExp2C0));
  uint32_t lo, hi;
  // bits(t) << 23 == n << 23 (the shift constant's low 9 bits are zero)
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(lo) : "r"(__float_as_uint(lo2(t))), "r"(__float_as_uint(lo2(q))));
  asm("mad.lo.u32 %0, %1, 8388608, %2;" : "=r"(hi) : "r"(__float_as_uint(hi2(t))), "r"(__float_as_uint(hi2(q))));
  return mk2(__uint_as_float(lo), __uint_as_float(hi));
}

// Pairs e of every 16-pair chunk whose exp2 runs on the FMA pipe (bit e of
// the mask); the others use the MUFU.  Two pairs of 16 (12.5 %, pairs 7 and
// 15) measured 2.5 % faster at CogVideoX-2B config 2 (0.915 against 0.938
// ms); four (25 %) no faster, eight (50 %) 10 % slower.
#ifndef SAF_EXP2_FMA_MASK
#define SAF_EXP2_FMA_MASK 0x8080u
#endif
__host__ __device__ constexpr bool exp2_on_fma(int e) { return (SAF_EXP2_FMA_MASK >> e) & 1u; }

// With a key bias, S = Q K^T + 1 b'^T: one more K = 16 MMA per tile whose A
// is a ones column (row m: [1, 0, ..., 0]) and whose B rows carry
// b'_j = bias_j / sm_scale in column 0 (16-bit, 32-byte swizzled tiles written
// by the producer warp).  Scaling S by sm_scale * log2(e) then adds
// bias_j * log2(e) to every logit, with no per-element work in the softmax.
template <int BN, bool kBias>
struct Layout {
  static constexpr int kQBytes = kBM * kD * 2;  // 16 KB
  static constexpr int kKVBytes = BN * kD * 2;  // 16 / 8 KB
  static constexpr int kBiasTile = BN * 32;     // BN rows x 16 16-bit values
  static constexpr int kOffQ = 0;
  static constexpr int kOffK = kOffQ + kQBytes;
  static constexpr int kOffV = kOffK + kKS * kKVBytes;
  static constexpr int kOffBias = kOffV + kVS * kKVBytes;          // [kVS] bias tiles
  static constexpr int kOffOnes = kOffBias + (kBias ? kVS * kBiasTile : 0);  // ones column
  static constexpr int kOffBar = kOffOnes + (kBias ? kBM * 32 : 0);
  // barriers: q_full, k_full[KS], k_empty[KS], v_full[VS], v_empty[VS],
  //           b_full[VS], s_full, s_empty, p_full, pv_full, drain, b_empty[VS],
  //           q_empty, tile_full[2], tile_empty[2], pool_full[2], pool_empty[2]
  static constexpr int kNumBars = 1 + 2 * kKS + 4 * kVS + 14;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  // tile lists (runtime size, after the fixed part): 2 slots of list_cap
  // uint16 entries, then two bitmaps of the key blocks
  static constexpr int kOffList = kOffMisc + 32;
  static constexpr int kBytes = kOffList;
  static constexpr int kDynSmem = kBytes + 1024;  // slack for 1024B alignment
};
inline int list_smem_bytes(int list_cap, int nbk) {
  return 2 * list_cap * 2 + 2 * ((nbk + 31) / 32) * 4 + 2 * 128 * 4;  // lists, bitmaps, pooled-map lse
}

// Masks applied inside a visited block, besides the ragged tail: none, the
// per-row key intervals of row_ranges, or the per-head frame masks.
constexpr int kMaskNone = 0, kMaskRanges = 1, kMaskFrames = 2;
// Key-list mode (no mask besides the ragged tail; K / V rows by gather4).
constexpr int kMaskKeys = 3;
// Attention with a pooled map (no mask besides the ragged tail).
constexpr int kMaskPool = 4;

// TMA gather4: four rows (coordinates r0..r3 of a 2-D map whose box is one
// row of 64 elements) into 4 x 128 bytes of shared memory, 128-byte swizzle
// applied as for a tile load.  No multicast.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int r0,
                                            int r1, int r2, int r3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(r0), "r"(r1), "r"(r2), "r"(r3)
      : "memory");
}

template <int BN, bool kBias, bool kBF16, int kMask>
__global__ void __launch_bounds__(kThreads, 2)
    bsa_fwd_sm100_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const BsaParams p) {
  using L = Layout<BN, kBias>;
  static_assert(kMask != kMaskKeys || (BN == 128 && !kBias), "key lists: 128-key blocks, no bias");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // Persistent CTAs: every CTA takes query tiles from a launch-wide counter
  // (the producer warp fetches them and hands them to the other roles through
  // a 2-slot ring in shared memory) until the counter passes the last tile.
  // Tile order: the first `lead_tiles` query tiles of every head (dense text
  // rows, the longest block lists) first, tile-major; the rest head-major so
  // that CTAs working at the same time share a head's K/V in L2.
  // A lead tile counts `splits` work items (consecutive), each a share of
  // its key blocks.  The split count is chosen here, the same in every CTA
  // (from the CSR's live-block total): a lead tile (about nbk blocks) is cut
  // so that no share exceeds the average work of a CTA, up to the host's cap.
  const int lead = p.lead_tiles < p.n_tiles ? p.lead_tiles : p.n_tiles;
  __shared__ int s_splits;
  if (warp == 0) {
    int sp = 1;
    if (p.splits > 1 && lead > 0) {
      long long nnz = 0;
      for (int gg = lane; gg < p.BH; gg += 32) {
        const int32_t* rp = p.row_ptr + static_cast<int64_t>(gg) * (p.nbq + 1);
        nnz += static_cast<long long>(max(0, rp[p.nbq] - rp[0]));
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) nnz += __shfl_xor_sync(0xffffffffu, nnz, off);
      const long long work = nnz * p.bm / kBM;  // blocks of 128-row tiles
      const long long want = work > 0 ? (static_cast<long long>(p.nbk) * gridDim.x + work - 1) / work : 1;
      sp = static_cast<int>(want < p.splits ? (want < 1 ? 1 : want) : p.splits);
    }
    if (lane == 0) s_splits = sp;
  }
  __syncthreads();
  const int n_split = s_splits;
  const int n_total = (lead * n_split + p.n_tiles - lead) * p.BH;
  auto tile_of = [&](int lin, int& tile, int& g, int& split) {
    if (lin < lead * p.BH * n_split) {
      split = lin % n_split;
      const int t2 = lin / n_split;
      tile = t2 / p.BH;
      g = t2 % p.BH;
    } else {
      const int rest = p.n_tiles - lead, l2 = lin - lead * p.BH * n_split;
      g = l2 / rest;
      tile = lead + l2 % rest;
      split = 0;
    }
  };
  const bool split_on = n_split > 1;

  const uint32_t sQ = smem_u32(smem + L::kOffQ);
  const uint32_t sK0 = smem_u32(smem + L::kOffK);
  const uint32_t sV0 = smem_u32(smem + L::kOffV);
  const uint32_t sBias0 = smem_u32(smem + L::kOffBias);
  const uint32_t sOnes = smem_u32(smem + L::kOffOnes);
  const uint32_t bar0 = smem_u32(smem + L::kOffBar);
  const uint32_t bar_q = bar0;
  auto bar_k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto bar_k_empty = [&](int s) { return bar0 + 8u * (1 + kKS + s); };
  auto bar_v_full = [&](int s) { return bar0 + 8u * (1 + 2 * kKS + s); };
  auto bar_v_empty = [&](int s) { return bar0 + 8u * (1 + 2 * kKS + kVS + s); };
  auto bar_b_full = [&](int s) { return bar0 + 8u * (1 + 2 * kKS + 2 * kVS + s); };
  auto bar_b_empty = [&](int s) { return bar0 + 8u * (1 + 2 * kKS + 3 * kVS + 5 + s); };
  const uint32_t bar_s_full = bar0 + 8u * (1 + 2 * kKS + 3 * kVS);
  const uint32_t bar_s_empty = bar_s_full + 8;
  const uint32_t bar_p_full = bar_s_full + 16;
  const uint32_t bar_pv_full = bar_s_full + 24;
  const uint32_t bar_drain = bar_s_full + 32;
  const uint32_t bar_q_empty = bar0 + 8u * (1 + 2 * kKS + 4 * kVS + 5);
  auto bar_tile_full = [&](int s) { return bar_q_empty + 8u * (1 + s); };
  auto bar_tile_empty = [&](int s) { return bar_q_empty + 8u * (3 + s); };
  // attention with a pooled map: the softmax warps hand each tile's block
  // maxima (in the scratch slot of the tile's parity) and the rows'
  // log2-sum-exp to warps 2-3, which pool them while the next tile runs
  auto bar_pool_full = [&](int s) { return bar_q_empty + 8u * (5 + s); };
  auto bar_pool_empty = [&](int s) { return bar_q_empty + 8u * (7 + s); };
  constexpr bool kPool = kMask == kMaskPool;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kOffMisc);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 4);
  volatile int* tile_slot = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 8);  // [2]
  volatile int* tile_cnt = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 16);  // [2] list lengths
  volatile int* tile_off = reinterpret_cast<volatile int*>(smem + L::kOffMisc + 24);  // [2] first list entry
  uint16_t* list_base = reinterpret_cast<uint16_t*>(smem + L::kOffList);            // [2][list_cap]
  uint32_t* list_bits = reinterpret_cast<uint32_t*>(smem + L::kOffList + 4 * p.list_cap);
  float* pool_lse = reinterpret_cast<float*>(list_bits + 2 * ((p.nbk + 31) / 32));  // [2][128]

  if (threadIdx.x == 0) {
    mbar_init(bar_q, 1);
    for (int s = 0; s < kKS; ++s) {
      mbar_init(bar_k_full(s), 1);
      mbar_init(bar_k_empty(s), 1);
    }
    for (int s = 0; s < kVS; ++s) {
      mbar_init(bar_v_full(s), 1);
      mbar_init(bar_v_empty(s), 1);
      mbar_init(bar_b_full(s), 32);
      mbar_init(bar_b_empty(s), 1);
    }
    mbar_init(bar_s_full, 1);
    mbar_init(bar_s_empty, 128);  // the softmax threads
    mbar_init(bar_p_full, 128);
    mbar_init(bar_pv_full, 1);
    mbar_init(bar_drain, 1);
    mbar_init(bar_q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(bar_tile_full(s), 1);
      // the MMA thread, the softmax threads and, pooling, warps 2-3
      mbar_init(bar_tile_empty(s), 1 + 128 + (kPool ? 64 : 0));
      mbar_init(bar_pool_full(s), 128);
      mbar_init(bar_pool_empty(s), 64);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  if constexpr (kBias) {
    // the ones column: 128 rows x 32 bytes, 32-byte swizzle (the 16-byte
    // half holding element 0 of row m is (m >> 2) & 1)
    const int m = threadIdx.x >> 1, half = threadIdx.x & 1;
    const uint32_t one = kBF16 ? 0x3F80u : 0x3C00u;
    const uint32_t w0 = half == ((m >> 2) & 1) ? one : 0u;
    st_shared_v4(sOnes + m * 32 + half * 16, w0, 0u, 0u, 0u);
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // Roles.  No code is shared after the register split: each warpgroup
  // ends with its own copy of the teardown (named barrier 1 over all
  // threads, then warp 1 frees TMEM).
  if (warp < 4) {
    setmaxnreg_dec<kRegsCtl>();
    if (warp == 0) {
    // ------------------------------------------------------------ producer
    int nk = 0, nv = 0, nq = 0, ti = 0, col;  // K / V / Q loads issued, tiles fetched
    bool ok = true;
    while (ok) {
      // next tile: fetched by lane 0, published in ring slot ti & 1
      int lin = 0;
      if (lane == 0) lin = static_cast<int>(atomicAdd(p.tile_ctr, 1u));
      lin = __shfl_sync(0xffffffffu, lin, 0);
      const int slot = ti & 1;
      ok = mbar_wait(bar_tile_empty(slot), ((ti >> 1) & 1) ^ 1, abort_flag, p.status, p.budget_ns);
      if (!__all_sync(0xffffffffu, ok)) break;
      int tile = 0, g = 0, split = 0, n_blk = 0, off = 0;
      uint16_t* lst = list_base + slot * p.list_cap;
      if (lin < n_total) {
        tile_of(lin, tile, g, split);
        n_blk = build_tile_list(p, g, tile, lst, list_bits, lane);
        if (split_on && tile < lead) {  // this item's share of the lead tile's blocks
          off = n_blk * split / n_split;
          n_blk = n_blk * (split + 1) / n_split - off;
        }
      }
      lst += off;
      __threadfence_block();
      __syncwarp();
      if (lane == 0) {
        tile_slot[slot] = lin;
        tile_cnt[slot] = n_blk;
        tile_off[slot] = off;
        mbar_arrive(bar_tile_full(slot));
      }
      __syncwarp();
      ++ti;
      if (lin >= n_total) break;
      const int b = g / p.H, h = g % p.H;
      // Q of this tile once the previous tile's QK^T products are done
      ok = mbar_wait(bar_q_empty, (nq & 1) ^ 1, abort_flag, p.status, p.budget_ns);
      if (!__all_sync(0xffffffffu, ok)) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(bar_q, L::kQBytes);
        tma_load_4d(sQ, &tm_q, bar_q, 0, tile * kBM, h, b);
      }
      ++nq;
      // key-list mode: this tile's list (the keys of its batch) and the row
      // base of its source head in the flat [B_src*H*S_src] row view of k / v;
      // each lane fetches four keys of a block, one block ahead of its loads
      const int32_t* kl = nullptr;
      int kbase = 0, knext[4] = {0, 0, 0, 0};
      auto fetch_keys = [&](int blk) {
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int jj = blk * BN + 4 * lane + u;
          knext[u] = jj < p.key_len ? kl[jj] : 0;  // rows past the list are masked in the softmax
        }
      };
      if constexpr (kMask == kMaskKeys) {
        int sb = p.key_batch[b];
        if (sb < 0 || sb >= p.key_src_batches) {
          atomicOr(p.status, SAF_DEV_BADINDEX);
          sb = 0;
        }
        kbase = (sb * p.H + h) * p.key_src_len;
        kl = p.key_list + static_cast<int64_t>(b) * p.key_len;
        if (n_blk > 0) fetch_keys(lst[0] & 0x3fff);
      }
      for (int jb = 0; jb < n_blk; ++jb) {
        col = lst[jb] & 0x3fff;
        const int sk = nk % kKS, sv = nv % kVS;
        const uint32_t pk = (nk / kKS) & 1, pv = (nv / kVS) & 1;
        int kr[4] = {0, 0, 0, 0};
        if constexpr (kMask == kMaskKeys) {
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            int kv = knext[u];
            if (kv < 0 || kv >= p.key_src_len) {
              atomicOr(p.status, SAF_DEV_BADINDEX);
              kv = 0;
            }
            kr[u] = kbase + kv;
          }
          if (jb + 1 < n_blk) fetch_keys(lst[jb + 1] & 0x3fff);  // in flight across this block's waits
        }
        // this block's key biases (loads in flight across the K-stage wait)
        float bvals[BN / 32];
        if constexpr (kBias) {
          const float* src = p.kv_bias + static_cast<int64_t>(g) * p.bias_stride;
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) {
            const int kv = col * BN + lane + 32 * i;
            bvals[i] = kv < p.Sk ? src[kv] : 0.f;
          }
        }
        ok = mbar_wait(bar_k_empty(sk), pk ^ 1, abort_flag, p.status, p.budget_ns);
        if (!__all_sync(0xffffffffu, ok)) break;
        if constexpr (kMask == kMaskKeys) {
          if (lane == 0) mbar_arrive_expect_tx(bar_k_full(sk), L::kKVBytes);
          __syncwarp();
          tma_gather4(sK0 + sk * L::kKVBytes + lane * 512, &tm_k, bar_k_full(sk), 0, kr[0], kr[1], kr[2], kr[3]);
        } else if (lane == 0) {
          mbar_arrive_expect_tx(bar_k_full(sk), L::kKVBytes);
          tma_load_4d(sK0 + sk * L::kKVBytes, &tm_k, bar_k_full(sk), 0, col * BN, h, b);
        }
        if constexpr (kBias) {
          // B rows of the bias MMA of block nk (its own 2-stage ring, freed by
          // that MMA's commit): key row c holds bias / sm_scale in element 0
          const int sb = nk % kVS;
          ok = mbar_wait(bar_b_empty(sb), ((nk / kVS) & 1) ^ 1, abort_flag, p.status, p.budget_ns);
          if (!__all_sync(0xffffffffu, ok)) break;
          const uint32_t dst = sBias0 + sb * L::kBiasTile;
#pragma unroll
          for (int i = 0; i < BN / 32; ++i) {
            const int c = lane + 32 * i;
            const float bv = bvals[i] * p.inv_scale;
            const uint32_t bits = kBF16 ? pack_bf16x2(bv, 0.f) : pack_f16x2(bv, 0.f);  // [bv, 0]
            const int hv = (c >> 2) & 1;
            st_shared_v4(dst + c * 32 + hv * 16, bits, 0u, 0u, 0u);
            st_shared_v4(dst + c * 32 + (hv ^ 1) * 16, 0u, 0u, 0u, 0u);
          }
          fence_proxy_async_smem();
          mbar_arrive(bar_b_full(sb));
        }
        ++nk;
        ok = mbar_wait(bar_v_empty(sv), pv ^ 1, abort_flag, p.status, p.budget_ns);
        if (!__all_sync(0xffffffffu, ok)) break;
        if constexpr (kMask == kMaskKeys) {
          if (lane == 0) mbar_arrive_expect_tx(bar_v_full(sv), L::kKVBytes);
          __syncwarp();
          tma_gather4(sV0 + sv * L::kKVBytes + lane * 512, &tm_v, bar_v_full(sv), 0, kr[0], kr[1], kr[2], kr[3]);
        } else if (lane == 0) {
          mbar_arrive_expect_tx(bar_v_full(sv), L::kKVBytes);
          tma_load_4d(sV0 + sv * L::kKVBytes, &tm_v, bar_v_full(sv), 0, col * BN, h, b);
        }
        ++nv;
      }
    }
    // Drain: wait for the last load issued into every stage (and so for all
    // earlier ones).  Immediate on the normal path, where the consumers have
    // already seen every load land.
    if (lane == 0) {
      if (nq > 0) mbar_drain(bar_q, (nq - 1) & 1, p.status);
      for (int s = 0; s < kKS && s < nk; ++s) {
        const int last = s + ((nk - 1 - s) / kKS) * kKS;
        mbar_drain(bar_k_full(s), (last / kKS) & 1, p.status);
      }
      for (int s = 0; s < kVS && s < nv; ++s) {
        const int last = s + ((nv - 1 - s) / kVS) * kVS;
        mbar_drain(bar_v_full(s), (last / kVS) & 1, p.status);
      }
    }
    __syncwarp();
    } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdescQK = idesc_f16(kBM, BN, kBF16, false, false);
      constexpr uint32_t kIdescPV = idesc_f16(kBM, kD, kBF16, false, true);
      const uint32_t tS = tmem + kColS, tO = tmem + kColO, tP = tmem + kColP;

      // O += P V for global block jg; `first` starts the tile's accumulator.
      auto issue_pv = [&](int jg, bool first) -> bool {
        const int sv = jg % kVS;
        const uint32_t pv = (jg / kVS) & 1;
        if (!mbar_wait(bar_v_full(sv), pv, abort_flag, p.status, p.budget_ns)) return false;
        if (!mbar_wait(bar_p_full, jg & 1, abort_flag, p.status, p.budget_ns)) return false;
        tc_fence_after();
        const uint32_t vbase = sV0 + sv * L::kKVBytes;
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          // B = V^T: N = D (contiguous, one 128B swizzle atom), K = kv rows;
          // 16 kv rows = two 8-row atoms = 2048 bytes.
          const uint64_t bdesc = sdesc_sw128(vbase + kk * 2048, L::kKVBytes, 1024);
          tc_mma_ts(tO, tP + kk * 8, bdesc, kIdescPV, (!first || kk > 0) ? 1u : 0u);
        }
        tc_commit(bar_pv_full);
        tc_commit(bar_v_empty(sv));
        return true;
      };

      int ti = 0, nq = 0, jbase = 0;  // tiles taken, Q tiles used, blocks of earlier tiles
      bool ok = true;
      while (ok) {
        const int slot = ti & 1;
        if (!mbar_wait(bar_tile_full(slot), (ti >> 1) & 1, abort_flag, p.status, p.budget_ns)) break;
        const int lin = tile_slot[slot];
        const int n_blk = tile_cnt[slot];  // the MMAs need only the block count
        mbar_arrive(bar_tile_empty(slot));
        ++ti;
        if (lin >= n_total) break;
        if (!mbar_wait(bar_q, nq & 1, abort_flag, p.status, p.budget_ns)) break;
        ++nq;
        tc_fence_after();
        int j = 0;  // blocks of this tile
        bool finished = false;
        while (true) {
          if (j >= n_blk) {
            finished = true;
            break;
          }
          const int jg = jbase + j;
          const int sk = jg % kKS;
          const uint32_t pk = (jg / kKS) & 1;
          if (!mbar_wait(bar_k_full(sk), pk, abort_flag, p.status, p.budget_ns)) break;
          if (!mbar_wait(bar_s_empty, (jg & 1) ^ 1, abort_flag, p.status, p.budget_ns)) break;
          tc_fence_after();
          const uint32_t kbase = sK0 + sk * L::kKVBytes;
#pragma unroll
          for (int kk = 0; kk < kD / 16; ++kk) {
            // K-major, 128B swizzle: 16 elements of K = 32 bytes along the row.
            const uint64_t adesc = sdesc_sw128(sQ + kk * 32, 16, 1024);
            const uint64_t bdesc = sdesc_sw128(kbase + kk * 32, 16, 1024);
            tc_mma_ss(tS, adesc, bdesc, kIdescQK, kk > 0 ? 1u : 0u);
          }
          if constexpr (kBias) {
            const int sb = jg % kVS;
            if (!mbar_wait(bar_b_full(sb), (jg / kVS) & 1, abort_flag, p.status, p.budget_ns)) break;
            tc_mma_ss(tS, sdesc_sw32(sOnes, 256), sdesc_sw32(sBias0 + sb * L::kBiasTile, 256), kIdescQK, 1u);
          }
          tc_commit(bar_s_full);
          tc_commit(bar_k_empty(sk));
          if constexpr (kBias) tc_commit(bar_b_empty(jg % kVS));
          if (j > 0 && !issue_pv(jg - 1, j == 1)) break;
          ++j;
        }
        // every QK^T of the tile is issued: Q is free once they complete
        tc_commit(bar_q_empty);
        if (!finished) {
          ok = false;
          break;
        }
        if (j > 0 && !issue_pv(jbase + j - 1, j == 1)) {
          ok = false;
          break;
        }
        jbase += j;
      }
      tc_commit(bar_drain);
      mbar_drain(bar_drain, 0, p.status);
    }
    } else if (kPool) {
    // ------------------------------------------------------------ pool reducer
    // Warps 2-3 (attention with a pooled map): for every tile, per listed
    // key block, exp2(R - lse) of each row, the maximum over a pool row
    // pooled into the map by an atomic max (non-negative floats order as
    // integers).  Thread t takes rows t and t + 64.
    const int t = threadIdx.x - 64;
    int ti = 0;
    while (true) {
      const int slot = ti & 1;
      const uint32_t par = (ti >> 1) & 1;
      if (!__all_sync(0xffffffffu, mbar_wait(bar_tile_full(slot), par, abort_flag, p.status, p.budget_ns))) break;
      const int lin = tile_slot[slot];
      const int n_blk = tile_cnt[slot];
      ++ti;
      if (lin >= n_total) {
        mbar_arrive(bar_tile_empty(slot));
        break;
      }
      int tile, g, split;
      tile_of(lin, tile, g, split);
      if (!__all_sync(0xffffffffu, mbar_wait(bar_pool_full(slot), par, abort_flag, p.status, p.budget_ns))) break;
      const float lse0 = pool_lse[slot * kBM + t], lse1 = pool_lse[slot * kBM + t + 64];
      const float* scr = p.pool_scratch + (static_cast<int64_t>(blockIdx.x) * 2 + slot) * p.list_cap * kBM;
      const uint16_t* lst = list_base + slot * p.list_cap;
      const int pr0 = tile * kBM / p.pool_block;
      int* po = reinterpret_cast<int*>(p.pool_out) + static_cast<int64_t>(g) * p.nbp * p.nbk;
      for (int j0 = 0; j0 < n_blk; j0 += 8) {
        float r0[8], r1[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int jj = j0 + u < n_blk ? j0 + u : n_blk - 1;
          r0[u] = scr[jj * kBM + t];
          r1[u] = scr[jj * kBM + t + 64];
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int jj = j0 + u;
          const float e0 = lse0 == -INFINITY ? 0.f : exp2f(r0[u] - lse0);
          const float e1 = lse1 == -INFINITY ? 0.f : exp2f(r1[u] - lse1);
          const int col = lst[jj < n_blk ? jj : 0] & 0x3fff;
          if (p.pool_block == kBM) {
            const uint32_t w = __reduce_max_sync(0xffffffffu, __float_as_uint(fmaxf(e0, e1)));
            if (lane == 0 && jj < n_blk && pr0 < p.nbp)
              atomicMax(po + static_cast<int64_t>(pr0) * p.nbk + col, static_cast<int>(w));
          } else {  // two pool rows of 64 per tile: rows t (first) and t + 64 (second)
            const uint32_t w0 = __reduce_max_sync(0xffffffffu, __float_as_uint(e0));
            const uint32_t w1 = __reduce_max_sync(0xffffffffu, __float_as_uint(e1));
            if (lane == 0 && jj < n_blk) {
              if (pr0 < p.nbp) atomicMax(po + static_cast<int64_t>(pr0) * p.nbk + col, static_cast<int>(w0));
              if (pr0 + 1 < p.nbp) atomicMax(po + static_cast<int64_t>(pr0 + 1) * p.nbk + col, static_cast<int>(w1));
            }
          }
        }
      }
      mbar_arrive(bar_pool_empty(slot));
      mbar_arrive(bar_tile_empty(slot));
    }
    }
    // ------------------------------------------------------------ teardown
    __syncwarp();
    tc_fence_before();
    named_barrier_sync(1, kThreads);
    if (warp == 1) {
      tc_fence_after();
      tmem_dealloc(tmem, kTmemCols);
    }
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ------------------------------------------------------------ softmax
    // One thread per query row holds the row's BN scores of a block, so the
    // block maximum needs no exchange between threads.
    constexpr int NC = BN / 32;  // 32-column TMEM chunks of a block
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    const uint32_t rhalf = static_cast<uint32_t>(row >> 6);  // row half (64-row mask blocks)
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_addr + kColS;
    const uint32_t tO = tmem + lane_addr + kColO;
    const uint32_t tP = tmem + lane_addr + kColP;
    const float sl2 = p.scale_log2;
    const f2 sl2x2 = mk2(sl2, sl2);

    int ti = 0, jbase = 0, col;  // tiles taken, blocks of earlier tiles
    uint32_t rm;
    bool ok = true;
    while (ok) {
    const int slot = ti & 1;
    if (!__all_sync(0xffffffffu, mbar_wait(bar_tile_full(slot), (ti >> 1) & 1, abort_flag, p.status,
                                            p.budget_ns))) {
      ok = false;
      break;
    }
    const int lin = tile_slot[slot];
    const int n_blk = tile_cnt[slot];
    ++ti;
    if (lin >= n_total) {
      mbar_arrive(bar_tile_empty(slot));
      break;
    }
    int tile, g, split;
    tile_of(lin, tile, g, split);
    const bool split_item = split_on && tile < lead;
    const int b = g / p.H, h = g % p.H;
    const int q0 = tile * kBM;
    float m_run = -INFINITY, l_run = 0.f;
    // key intervals of this thread's query row (kMaskRanges)
    int lo0 = 0, hi0 = 0, lo1 = 0, hi1 = 0;
    if constexpr (kMask == kMaskRanges) {
      if (q0 + row < p.Sq) {
        const int4 rr = __ldg(p.row_ranges + q0 + row);
        lo0 = rr.x, hi0 = rr.y, lo1 = rr.z, hi1 = rr.w;
      }
    }
    // key frames this thread's query row may see (kMaskFrames): all for a
    // text row, the head's mask word of the row's frame for a video row
    uint32_t fbits = 0xffffffffu;
    if constexpr (kMask == kMaskFrames) {
      const int qr = q0 + row;
      if (qr >= p.Sq) {
        fbits = 0u;
      } else if (qr >= p.text_len) {
        const int fq = (qr - p.text_len) / p.frame_len;
        fbits = __ldg(p.frame_bits + static_cast<int64_t>(g) * p.frames + fq);
      }
    }
    const uint16_t* lst = list_base + slot * p.list_cap + tile_off[slot];
    if constexpr (kPool) {
      // this parity's scratch slot is free once the reducer pooled the tile
      // two tiles back
      if (!__all_sync(0xffffffffu, mbar_wait(bar_pool_empty(slot), (((ti - 1) >> 1) & 1) ^ 1, abort_flag,
                                              p.status, p.budget_ns))) {
        ok = false;
        break;
      }
    }
    int j = 0;  // blocks of this tile
    while (j < n_blk) {
      const uint32_t ent = lst[j];
      col = static_cast<int>(ent & 0x3fffu);
      rm = ent >> 14;
      const int jg = jbase + j;
      if (!__all_sync(0xffffffffu,
                      mbar_wait(bar_s_full, jg & 1, abort_flag, p.status, p.budget_ns))) {
        ok = false;
        break;
      }
      tc_fence_after();
      // x32 loads (no single instruction may need more registers than the
      // launch budget); one wait covers all of them.
      uint32_t r[NC][32];
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_ld32(tS + 32 * c, r[c]);
#pragma unroll
      for (int c = 0; c < NC; ++c) tmem_wait_ld(r[c]);
      // The row's scores are in registers: the next QK^T may overwrite S.
      tc_fence_before();
      mbar_arrive(bar_s_empty);

      const bool live = (rm >> rhalf) & 1u;
      const int c0 = col * BN;      // first key column of the block
      const int valid = p.Sk - c0;  // valid columns of the block
      bool fast = live && valid >= BN;
      if constexpr (kMask == kMaskRanges)
        fast = fast && ((c0 >= lo0 && c0 + BN <= hi0) || (c0 >= lo1 && c0 + BN <= hi1));
      // kMaskFrames: the block's keys are [c0, c0 + bnd) of region a and
      // [c0 + bnd, c0 + BN) of region b (one frame boundary at most: frames
      // are at least BN keys long); a region is text (-1) or a frame
      bool ok_a = true, ok_b = true;
      int bnd = BN;
      if constexpr (kMask == kMaskFrames) {
        const int T = p.text_len, FL = p.frame_len;
        const int cl = (valid < BN ? p.Sk : c0 + BN) - 1;  // last key of the block
        const int ka = c0 < T ? -1 : (c0 - T) / FL;
        const int kb = cl < T ? -1 : (cl - T) / FL;
        if (kb != ka) bnd = T + kb * FL - c0;
        ok_a = ka < 0 || ((fbits >> ka) & 1u);
        ok_b = kb < 0 || ((fbits >> kb) & 1u);
        fast = fast && ok_a && ok_b;
      }
      // (a key bias is already in S: see Layout)
      float t[BN];
#pragma unroll
      for (int e = 0; e < BN; ++e) t[e] = __uint_as_float(r[e / 32][e % 32]);
      if (!fast) {
        if constexpr (kMask == kMaskFrames) {
#pragma unroll
          for (int e = 0; e < BN; ++e)
            if (!(live && e < valid && (e < bnd ? ok_a : ok_b))) t[e] = -INFINITY;
        } else if constexpr (kMask == kMaskRanges) {
          const int a0 = lo0 - c0, b0 = hi0 - c0, a1 = lo1 - c0, b1 = hi1 - c0;
#pragma unroll
          for (int e = 0; e < BN; ++e)
            if (!(live && e < valid && ((e >= a0 && e < b0) || (e >= a1 && e < b1)))) t[e] = -INFINITY;
        } else {
#pragma unroll
          for (int e = 0; e < BN; ++e)
            if (!(live && e < valid)) t[e] = -INFINITY;
        }
      }
      // Under lazy rescaling the running max rarely moves, so P is computed
      // speculatively with the current running max while the block max is
      // accumulated alongside (ALU work next to the MUFU work); only if the
      // row's max jumped past the threshold does the warp recompute P (the
      // scores are still in registers) and rescale O.  A warp with a row that
      // has not seen a live score yet takes the max-first order.
      const bool spec = __all_sync(0xffffffffu, m_run != -INFINITY);
      bool pv_done = (j == 0);
      // PV of the previous block must be done before P is overwritten and
      // before O is rescaled.
      auto wait_pv = [&]() -> bool {
        if (pv_done) return true;
        if (!__all_sync(0xffffffffu, mbar_wait(bar_pv_full, (jg - 1) & 1, abort_flag, p.status,
                                                p.budget_ns)))
          return false;
        tc_fence_after();
        pv_done = true;
        return true;
      };
      f2 rs = mk2(0.f, 0.f);
      float mx = -INFINITY;
      // P = exp2(logit - m) in the input type, row sum in fp32 pairs, 32
      // scores at a time (the empty asm after each store keeps the next part's
      // exp2 from being scheduled early, bounding live registers).
      // zero: P of a row with no live score yet is 0 (the polynomial maps
      // -inf to 2^-126, not 0), keeping such rows at l = 0 as the reference.
      auto exp_pass = [&](float neg_m, bool with_max, bool zero) -> bool {
        const f2 negm2 = mk2(neg_m, neg_m);
        rs = mk2(0.f, 0.f);
        float acc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (with_max)
              acc[e & 3] = fmax3(acc[e & 3], t[c * 32 + 2 * e], t[c * 32 + 2 * e + 1]);
            f2 x = mk2(t[c * 32 + 2 * e], t[c * 32 + 2 * e + 1]);
            x = fma2(x, sl2x2, negm2);
            float e0, e1;
            if (exp2_on_fma(e)) {
              const f2 y = exp2_poly2(x);
              e0 = lo2(y);
              e1 = hi2(y);
            } else {
              e0 = ex2_approx(lo2(x));
              e1 = ex2_approx(hi2(x));
            }
            if (zero) {
              e0 = 0.f;
              e1 = 0.f;
            }
            rs = add2(rs, mk2(e0, e1));
            pk[e] = kBF16 ? pack_bf16x2(e0, e1) : pack_f16x2(e0, e1);
          }
          if (c == 0 && !wait_pv()) return false;
          tmem_st16(tP + c * 16, pk);
          if (c + 1 < NC) {
            asm volatile("" : "+l"(rs.v));
#pragma unroll
            for (int e = 0; e < 32; ++e) asm volatile("" : "+f"(t[(c + 1) * 32 + e]));
          }
        }
        if (with_max) mx = fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3]));
        return true;
      };

      auto block_max = [&]() {
        float acc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int i = 0; i < BN / 2; ++i) acc[i & 3] = fmax3(acc[i & 3], t[2 * i], t[2 * i + 1]);
        return fmaxf(fmaxf(acc[0], acc[1]), fmaxf(acc[2], acc[3]));
      };
#if SAF_OVERFLOW_GUARD
      // Speculative P with the running max, no block maximum: the max moves
      // only for a row whose block sum shows P could approach overflow
      // (> 2^64; the normalised result does not depend on which max P was
      // taken against).  The pooled map needs every block's maximum, so that
      // mode keeps the threshold rule below.
      constexpr bool kGuard = kMask != kMaskPool;
#else
      constexpr bool kGuard = false;
#endif
      if (spec) {
        if (!exp_pass(-m_run, !kGuard, false)) {
          ok = false;
          break;
        }
      } else {
        mx = block_max();
      }
      bool upd;
      if (kGuard && spec) {
        upd = !(lo2(rs) + hi2(rs) <= 1.8446744e19f);  // 2^64; catches inf and NaN too
        if (__any_sync(0xffffffffu, upd)) mx = block_max() * sl2;
      } else {
        mx *= sl2;
        upd = mx > m_run + kRescaleThreshold;
      }
      if constexpr (kPool)
        p.pool_scratch[((static_cast<int64_t>(blockIdx.x) * 2 + slot) * p.list_cap + j) * kBM + row] = mx;
      const float m_new = upd ? mx : m_run;
      const float alpha = upd ? ex2_approx(m_run - m_new) : 1.f;
      const float neg_m = (m_new == -INFINITY) ? 0.f : -m_new;
      const bool any_upd = __any_sync(0xffffffffu, upd);
      if (!spec || any_upd) {
        if (!exp_pass(neg_m, false, m_new == -INFINITY)) {
          ok = false;
          break;
        }
      }
      if (j > 0 && any_upd) {
        if (!wait_pv()) {
          ok = false;
          break;
        }
#pragma unroll
        for (int c = 0; c < kD / 32; ++c) {
          uint32_t orr[32];
          tmem_ld32(tO + 32 * c, orr);
          tmem_wait_ld(orr);
#pragma unroll
          for (int e = 0; e < 32; ++e) orr[e] = __float_as_uint(__uint_as_float(orr[e]) * alpha);
          tmem_st32(tO + 32 * c, orr);
        }
      }
      l_run = l_run * alpha + (lo2(rs) + hi2(rs));
      m_run = m_new;
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(bar_p_full);
      ++j;
    }
    // ---------------------------------------------------------- epilogue
    // O is read back 32 columns at a time, normalised by 1/l and stored.  A
    // zero row sum gives 0 * inf = NaN, matching the reference; a tile with no
    // live block never wrote O and stores NaN as well.
    const bool have_o =
        ok && j > 0 &&
        __all_sync(0xffffffffu,
                   mbar_wait(bar_pv_full, (jbase + j - 1) & 1, abort_flag, p.status, p.budget_ns));
    if (have_o) tc_fence_after();
    const int qrow = q0 + row;
    const float inv_l = 1.f / l_run;
    if constexpr (kPool) {
      // hand the tile's row statistics to the pool reducer (warps 2-3); a
      // row past Sq or with no visible key pools nothing
      pool_lse[slot * kBM + row] = (ok && qrow < p.Sq && l_run > 0.f) ? m_run + log2f(l_run) : -INFINITY;
      mbar_arrive(bar_pool_full(slot));
    }
    uint8_t* dst = reinterpret_cast<uint8_t*>(p.o) +
                   2 * (static_cast<int64_t>(b) * p.o_sb + static_cast<int64_t>(h) * p.o_sh +
                        static_cast<int64_t>(qrow) * p.o_ss);
    auto store_row = [&](const float* vals, float scale) {
#pragma unroll
      for (int v = 0; v < kD / 8; ++v) {
        uint4 w;
        uint32_t* pw = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = vals[v * 8 + 2 * e] * scale, hi = vals[v * 8 + 2 * e + 1] * scale;
          pw[e] = kBF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
        }
        reinterpret_cast<uint4*>(dst)[v] = w;
      }
    };
    if (split_item) {
      // a share of a lead tile: the row's unnormalised O, m and l go to the
      // split buffer; the last share of the row to finish merges them all
      float* part = p.split_part +
                    ((((static_cast<int64_t>(g) * lead + tile) * n_split + split) * kBM) + row) * kSplitRow;
#pragma unroll
      for (int c = 0; c < kD / 32; ++c) {
        uint32_t orr[32];
        if (have_o) {
          tmem_ld32(tO + 32 * c, orr);
          tmem_wait_ld(orr);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) orr[e] = 0u;
        }
#pragma unroll
        for (int v = 0; v < 8; ++v)
          reinterpret_cast<float4*>(part)[c * 8 + v] =
              make_float4(__uint_as_float(orr[4 * v]), __uint_as_float(orr[4 * v + 1]),
                          __uint_as_float(orr[4 * v + 2]), __uint_as_float(orr[4 * v + 3]));
      }
      part[kD] = m_run;
      part[kD + 1] = (have_o || j == 0) ? l_run : 0.f;
      __threadfence();
      int* cnt = p.split_cnt + (static_cast<int64_t>(g) * lead + tile) * kBM + row;
      if (atomicAdd(cnt, 1) == n_split - 1) {
        __threadfence();
        const float* base = p.split_part + (((static_cast<int64_t>(g) * lead + tile) * n_split) * kBM + row) * kSplitRow;
        const int64_t sstride = static_cast<int64_t>(kBM) * kSplitRow;
        float mm = -INFINITY;
        for (int sp = 0; sp < n_split; ++sp) {
          const float ls = __ldcg(base + sp * sstride + kD + 1);
          if (ls > 0.f) mm = fmaxf(mm, __ldcg(base + sp * sstride + kD));
        }
        float acc[kD];
#pragma unroll
        for (int d = 0; d < kD; ++d) acc[d] = 0.f;
        float ll = 0.f;
        for (int sp = 0; sp < n_split; ++sp) {
          const float* ps = base + sp * sstride;
          const float ls = __ldcg(ps + kD + 1);
          if (!(ls > 0.f)) continue;
          const float wgt = ex2_approx(__ldcg(ps + kD) - mm);
          ll += ls * wgt;
#pragma unroll
          for (int d4 = 0; d4 < kD / 4; ++d4) {
            const float4 o4 = __ldcg(reinterpret_cast<const float4*>(ps) + d4);
            acc[4 * d4] += o4.x * wgt;
            acc[4 * d4 + 1] += o4.y * wgt;
            acc[4 * d4 + 2] += o4.z * wgt;
            acc[4 * d4 + 3] += o4.w * wgt;
          }
        }
        *cnt = 0;
        // no visible key in any share: 0 / 0 = NaN, as the unsplit path
        if (ok && !*abort_flag && qrow < p.Sq) store_row(acc, 1.f / ll);
      }
    } else {
    const bool write = (j == 0 || have_o) && ok && !*abort_flag && qrow < p.Sq;
#pragma unroll
    for (int c = 0; c < kD / 32; ++c) {
      uint32_t orr[32];
      if (have_o) {
        tmem_ld32(tO + 32 * c, orr);
        tmem_wait_ld(orr);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) orr[e] = 0u;
      }
      if (write) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint4 w;
          uint32_t* pw = reinterpret_cast<uint32_t*>(&w);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = __uint_as_float(orr[v * 8 + 2 * e]) * inv_l;
            const float hi = __uint_as_float(orr[v * 8 + 2 * e + 1]) * inv_l;
            pw[e] = kBF16 ? pack_bf16x2(lo, hi) : pack_f16x2(lo, hi);
          }
          reinterpret_cast<uint4*>(dst)[c * 4 + v] = w;
        }
      }
    }
    }
    // the tile's block list is no longer read: the producer may refill the slot
    mbar_arrive(bar_tile_empty(slot));
    jbase += j;
    }  // tile loop
    tc_fence_before();
    named_barrier_sync(1, kThreads);
  }
  // The last CTA to finish resets this launch's tile counters.
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.tile_ctr + 1, 1u) == gridDim.x - 1) {
      p.tile_ctr[0] = 0u;
      p.tile_ctr[1] = 0u;
      __threadfence();
    }
  }
}

// Tile counters of the persistent schedule: 64 launch slots of [next tile,
// CTAs done] per device, taken round-robin by the launches (a launch leaves
// its slot at zero when its last CTA exits, so launches 64 apart -- or
// ordered on one stream -- never share a live slot).
__device__ unsigned int g_tile_ctr[64 * 2];
constexpr int kMaxDevices = 64;
std::atomic<unsigned int> g_launch_seq{0};
unsigned int* g_ctr_base[kMaxDevices] = {};

int32_t tile_counter_slot(unsigned int** out) {
  int dev = 0;
  SAF_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return SAF_ERR_UNSUPPORTED;
  if (g_ctr_base[dev] == nullptr) {
    void* ptr = nullptr;
    SAF_CUDA_TRY(cudaGetSymbolAddress(&ptr, g_tile_ctr));
    g_ctr_base[dev] = static_cast<unsigned int*>(ptr);
  }
  *out = g_ctr_base[dev] + 2 * (g_launch_seq.fetch_add(1u) % 64u);
  return SAF_OK;
}

// Split buffers of the lead tiles (static per device, like the tile
// counters): partial rows [heads x lead tiles x splits x 128 x 66] fp32 and
// one counter per (head, lead tile, row).  A launch whose split buffers would
// not fit runs its lead tiles unsplit.
constexpr int64_t kSplitFloats = int64_t(4) << 20;  // 16 MiB
constexpr int64_t kSplitCnts = int64_t(1) << 18;    // 1 MiB
__device__ __align__(16) float g_split_part[kSplitFloats];
__device__ int g_split_cnt[kSplitCnts];
float* g_split_part_base[kMaxDevices] = {};
int* g_split_cnt_base[kMaxDevices] = {};

int32_t split_buffers(float** part, int** cnt) {
  int dev = 0;
  SAF_CUDA_TRY(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kMaxDevices) return SAF_ERR_UNSUPPORTED;
  if (g_split_part_base[dev] == nullptr) {
    void* a = nullptr;
    void* c = nullptr;
    SAF_CUDA_TRY(cudaGetSymbolAddress(&a, g_split_part));
    SAF_CUDA_TRY(cudaGetSymbolAddress(&c, g_split_cnt));
    g_split_cnt_base[dev] = static_cast<int*>(c);
    g_split_part_base[dev] = static_cast<float*>(a);
  }
  *part = g_split_part_base[dev];
  *cnt = g_split_cnt_base[dev];
  return SAF_OK;
}

template <int BN, bool kBias, bool kBF16, int kMask>
int32_t launch_variant(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                       BsaParams p, int n_tiles, cudaStream_t stream) {
  auto kern = bsa_fwd_sm100_kernel<BN, kBias, kBF16, kMask>;
  p.list_cap = (p.nbk + 7) / 8 * 8;
  const int smem = Layout<BN, kBias>::kDynSmem + list_smem_bytes(p.list_cap, p.nbk);
  SAF_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
  // setmaxnreg.inc only draws on the registers the CTA was launched with: a
  // build that launched with fewer than the split needs would wait forever
  static const int launch_regs = [] {
    cudaFuncAttributes fa{};
    return cudaFuncGetAttributes(&fa, bsa_fwd_sm100_kernel<BN, kBias, kBF16, kMask>) == cudaSuccess ? fa.numRegs
                                                                                                  : 0;
  }();
  if (launch_regs * kThreads < 128 * static_cast<int>(kRegsCtl + kRegsSoftmax)) return SAF_ERR_UNSUPPORTED;
  int dev = 0, sms = 0;
  SAF_CUDA_TRY(cudaGetDevice(&dev));
  SAF_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  int32_t rc = tile_counter_slot(&p.tile_ctr);
  if (rc != SAF_OK) return rc;
  p.n_tiles = n_tiles;
  p.BH = p.B * p.H;
  // Lead tiles (dense text rows: every key block) are the longest work items;
  // with few heads per GPU a single one outlasts the rest of the launch, so
  // their key blocks may be split over several items.  The host sets the cap
  // (buffer capacity, at most 8); the kernel picks the count from the CSR.
  // The grid is sized for the cap; CTAs without an item return at once.
  const int lead = p.lead_tiles < n_tiles ? p.lead_tiles : n_tiles;
  p.splits = 1;
  if (lead > 0 && kMask != kMaskPool && kMask != kMaskKeys) {
    const int64_t items = static_cast<int64_t>(lead) * p.BH;
    int sp = static_cast<int>(std::min<int64_t>(8, (2 * sms + items - 1) / items));
    if (sp > 1 && items * sp * kBM * kSplitRow <= kSplitFloats && items * kBM <= kSplitCnts) {
      if ((rc = split_buffers(&p.split_part, &p.split_cnt)) != SAF_OK) return rc;
      SAF_CUDA_TRY(cudaMemsetAsync(p.split_cnt, 0, static_cast<size_t>(items * kBM) * sizeof(int), stream));
      p.splits = sp;
    }
  }
  const int64_t total = (static_cast<int64_t>(lead) * p.splits + n_tiles - lead) * p.BH;
  const int grid = static_cast<int>(total < 2 * sms ? total : 2 * sms);  // two CTAs per SM
  kern<<<grid, kThreads, smem, stream>>>(mq, mk, mv, p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

}  // namespace

// Host entry for 16-bit inputs (validated by the caller in saf_api.cu).
int32_t bsa_fwd_sm100(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                      const saf_tensor4* o, const int32_t* row_ptr, const int32_t* col_idx,
                      int64_t col_capacity, int bm, int bn, const float* kv_bias,
                      int64_t bias_stride, float sm_scale, int lead_tiles, const int32_t* row_ranges,
                      const FrameMaskArgs* frames, const PoolArgs* pool,
                      cudaStream_t stream) {
  if (q->D != kD) return SAF_ERR_UNSUPPORTED;
  if (frames != nullptr && (row_ranges != nullptr || kv_bias != nullptr)) return SAF_ERR_UNSUPPORTED;
  if (row_ranges != nullptr && kv_bias != nullptr) return SAF_ERR_UNSUPPORTED;
  if (!current_device_is_sm100()) return SAF_ERR_UNSUPPORTED;
  CUtensorMap mq, mk, mv;
  int32_t rc;
  if ((rc = make_qkv_map(&mq, q, kBM)) != SAF_OK) return rc;
  if ((rc = make_qkv_map(&mk, k, bn)) != SAF_OK) return rc;
  if ((rc = make_qkv_map(&mv, v, bn)) != SAF_OK) return rc;
  BsaParams p{};
  p.B = static_cast<int>(q->B);
  p.H = static_cast<int>(q->H);
  p.Sq = static_cast<int>(q->S);
  p.Sk = static_cast<int>(k->S);
  p.bm = bm;
  p.nbq = static_cast<int>((q->S + bm - 1) / bm);
  p.nbk = static_cast<int>((k->S + bn - 1) / bn);
  if (p.nbk > 16384) return SAF_ERR_UNSUPPORTED;  // 14-bit columns in the tile lists
  p.col_capacity = col_capacity;
  p.row_ptr = row_ptr;
  p.col_idx = col_idx;
  p.kv_bias = kv_bias;
  p.bias_stride = bias_stride;
  p.scale_log2 = sm_scale * kLog2e;
  p.inv_scale = static_cast<float>(1.0 / static_cast<double>(sm_scale));
  p.o = o->data;
  p.o_sb = o->stride_b;
  p.o_sh = o->stride_h;
  p.o_ss = o->stride_s;
  p.status = device_status_ptr();
  p.budget_ns = wait_budget_ns();
  p.lead_tiles = lead_tiles;
  p.row_ranges = reinterpret_cast<const int4*>(row_ranges);
  if (frames != nullptr) {
    p.frame_bits = frames->bits;
    p.text_len = frames->text_len;
    p.frame_len = frames->frame_len;
    p.frames = frames->frames;
  }
  if (pool != nullptr) {
    p.pool_scratch = pool->scratch;
    p.pool_out = pool->out;
    p.pool_block = pool->pool_block;
    p.nbp = static_cast<int>((q->S + pool->pool_block - 1) / pool->pool_block);
  }
  if (p.status == nullptr) return SAF_ERR_CUDA;
  const int n_tiles = static_cast<int>((q->S + kBM - 1) / kBM);
  const bool bf16 = q->dtype == SAF_BF16;
  const bool bias = kv_bias != nullptr;
  const int mask = frames != nullptr ? kMaskFrames
                   : row_ranges != nullptr ? kMaskRanges
                   : pool != nullptr       ? kMaskPool
                                           : kMaskNone;
  if (pool != nullptr && (bias || frames != nullptr || row_ranges != nullptr)) return SAF_ERR_UNSUPPORTED;
#define SAF_BSA_CASE(BN_, BIAS_, BF_, MASK_)                               \
  if (bn == BN_ && bias == BIAS_ && bf16 == BF_ && mask == MASK_)          \
    return launch_variant<BN_, BIAS_, BF_, MASK_>(mq, mk, mv, p, n_tiles, stream);
  SAF_BSA_CASE(128, false, true, kMaskNone)
  SAF_BSA_CASE(128, true, true, kMaskNone)
  SAF_BSA_CASE(128, false, false, kMaskNone)
  SAF_BSA_CASE(128, true, false, kMaskNone)
  SAF_BSA_CASE(64, false, true, kMaskNone)
  SAF_BSA_CASE(64, true, true, kMaskNone)
  SAF_BSA_CASE(64, false, false, kMaskNone)
  SAF_BSA_CASE(64, true, false, kMaskNone)
  SAF_BSA_CASE(128, false, true, kMaskRanges)
  SAF_BSA_CASE(128, false, false, kMaskRanges)
  SAF_BSA_CASE(64, false, true, kMaskRanges)
  SAF_BSA_CASE(64, false, false, kMaskRanges)
  SAF_BSA_CASE(128, false, true, kMaskFrames)
  SAF_BSA_CASE(128, false, false, kMaskFrames)
  SAF_BSA_CASE(64, false, true, kMaskFrames)
  SAF_BSA_CASE(64, false, false, kMaskFrames)
  SAF_BSA_CASE(128, false, true, kMaskPool)
  SAF_BSA_CASE(128, false, false, kMaskPool)
  SAF_BSA_CASE(64, false, true, kMaskPool)
  SAF_BSA_CASE(64, false, false, kMaskPool)
#undef SAF_BSA_CASE
  return SAF_ERR_UNSUPPORTED;
}

// Host entry of the key-list mode: q / o [Bq, H, Sq, 64], k / v
// [B_src, H, S_src, 64] with contiguous rows, key_list [Bq, key_len] int32
// (keys of k[key_batch[b]]), every key block live.
int32_t bsa_fwd_sm100_keys(const saf_tensor4* q, const saf_tensor4* k, const saf_tensor4* v,
                           const saf_tensor4* o, const int32_t* key_list, int32_t key_len,
                           const int32_t* key_batch, float sm_scale, cudaStream_t stream) {
  if (q->D != kD || k->D != kD) return SAF_ERR_UNSUPPORTED;
  if (q->dtype != SAF_BF16 && q->dtype != SAF_F16) return SAF_ERR_UNSUPPORTED;
  if (!current_device_is_sm100()) return SAF_ERR_UNSUPPORTED;
  for (const saf_tensor4* t : {k, v})
    if (t->stride_s != kD || t->stride_h != t->S * kD || (t->B > 1 && t->stride_b != t->H * t->S * kD))
      return SAF_ERR_STRIDE;  // the gather reads k / v as one array of 64-element rows
  const int64_t rows = k->B * k->H * k->S;
  if (rows >= (int64_t(1) << 31) || key_len <= 0) return SAF_ERR_SHAPE;
  CUtensorMap mq, mk, mv;
  int32_t rc;
  if ((rc = make_qkv_map(&mq, q, kBM)) != SAF_OK) return rc;
  const CUtensorMapDataType dt =
      q->dtype == SAF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  for (int t = 0; t < 2; ++t) {
    const saf_tensor4* src = t == 0 ? k : v;
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(kD), static_cast<cuuint64_t>(rows)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(kD * 2)};
    cuuint32_t box[2] = {static_cast<cuuint32_t>(kD), 1u};  // one row: the gather4 box
    if (encode_tensor_map(t == 0 ? &mk : &mv, dt, 2, src->data, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B) !=
        CUDA_SUCCESS)
      return SAF_ERR_STRIDE;
  }
  BsaParams p{};
  p.B = static_cast<int>(q->B);
  p.H = static_cast<int>(q->H);
  p.Sq = static_cast<int>(q->S);
  p.Sk = key_len;
  p.bm = 128;
  p.nbq = static_cast<int>((q->S + kBM - 1) / kBM);
  p.nbk = (key_len + 127) / 128;
  if (p.nbk > 16384) return SAF_ERR_UNSUPPORTED;
  p.dense = 1;
  p.scale_log2 = sm_scale * kLog2e;
  p.inv_scale = static_cast<float>(1.0 / static_cast<double>(sm_scale));
  p.o = o->data;
  p.o_sb = o->stride_b;
  p.o_sh = o->stride_h;
  p.o_ss = o->stride_s;
  p.status = device_status_ptr();
  p.budget_ns = wait_budget_ns();
  p.key_list = key_list;
  p.key_batch = key_batch;
  p.key_len = key_len;
  p.key_src_len = static_cast<int>(k->S);
  p.key_src_batches = static_cast<int>(k->B);
  if (p.status == nullptr) return SAF_ERR_CUDA;
  const int n_tiles = p.nbq;
  if (q->dtype == SAF_BF16) return launch_variant<128, false, true, kMaskKeys>(mq, mk, mv, p, n_tiles, stream);
  return launch_variant<128, false, false, kMaskKeys>(mq, mk, mv, p, n_tiles, stream);
}

}  // namespace saf
