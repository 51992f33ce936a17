// Ulysses layout kernels: pack a sequence shard into per-peer head chunks
// for the sequence -> head all-to-all, and unpack the chunks received on the
// way back.
//
// Sequence-sharded tensors are [B, s, H, D] (the layout of a q/k/v
// projection of a sequence shard; any strides with D contiguous).  The
// exchange buffer holds P chunks back to back; chunk j carries heads
// [head_off[j], head_off[j+1]) of T tensors as [s, B, T, h_j, D], so that
// after the all-to-all the receiver's buffer is [S, B, T, h, D] for its own
// heads: sequence-major, and each tensor of it is the strided
// [B, h, S, D] view the attention kernels read directly (no unpack on the
// forward path).  The return path sends [s_i, B, h, D] rows of the
// attention output and unpacks the received [s, B, 1, h_j, D] chunks into
// [B, s, H, D].
//
// One thread per 16-byte vector of a D row; D * element size must be a
// multiple of 16 bytes and every row start 16-byte aligned (host-checked).
#include <algorithm>
#include <cstdint>

#include "saf_common.cuh"

namespace saf {
namespace {

constexpr int kMaxPeers = 64;
constexpr int kMaxTensors = 4;

struct UlyssesParams {
  void* seq[kMaxTensors];    // T sequence-sharded tensors [B, s, H, D]
  void* buf;                 // exchange buffer (P chunks)
  int64_t s_b, s_s, s_h;     // element strides of the sequence-sharded tensors
  int64_t chunk_off[kMaxPeers + 1];  // element offset of chunk j in buf
  int32_t head_off[kMaxPeers + 1];
  int32_t T, B, s, D, vec;   // vec = 16-byte vectors per D row
};

// kPack: seq -> buf; otherwise buf -> seq.  A chunk row is one (s, b) pair
// of T * h_j * vec 16-byte vectors, contiguous in buf.  threadIdx.x fixes a
// thread's (t, h, vector) positions within a row for the whole launch (the
// only divisions by T, h_j and vec), threadIdx.y and the grid-stride loop
// pick rows; consecutive lanes cover consecutive vectors of buf and of a D
// row, so both sides stay coalesced.
template <bool kPack>
__global__ void __launch_bounds__(1024) ulysses_copy_kernel(const UlyssesParams p) {
  const int j = blockIdx.y;
  const int hj = p.head_off[j + 1] - p.head_off[j];
  const int inner = p.T * hj * p.vec;
  const int64_t elem_bytes = 16LL * p.vec / p.D;  // vec = D * element size / 16
  const int64_t sb_v = p.s_b * elem_bytes / 16, ss_v = p.s_s * elem_bytes / 16;  // strides in vectors
  const int rows = p.s * p.B;
  uint4* buf0 = reinterpret_cast<uint4*>(static_cast<char*>(p.buf) + p.chunk_off[j] * elem_bytes);
  for (int i = threadIdx.x; i < inner; i += blockDim.x) {
    const int v = i % p.vec;
    const int th = i / p.vec;
    const int h = th % hj;
    const int t = th / hj;
    uint4* seq0 = reinterpret_cast<uint4*>(static_cast<char*>(p.seq[t]) +
                                           static_cast<int64_t>(p.head_off[j] + h) * p.s_h * elem_bytes) + v;
    // four rows per step: four independent loads in flight per thread
    const int stride = gridDim.x * blockDim.y;
    for (int row0 = blockIdx.x * blockDim.y + threadIdx.y; row0 < rows; row0 += 4 * stride) {
      uint4 val[4];
      uint4* dst[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int row = row0 + u * stride;
        dst[u] = nullptr;
        if (row < rows) {
          const int s = row / p.B, b = row - s * p.B;
          uint4* bv = buf0 + static_cast<int64_t>(row) * inner + i;
          uint4* sv = seq0 + b * sb_v + s * ss_v;
          if constexpr (kPack) {
            val[u] = __ldg(sv);
            dst[u] = bv;
          } else {
            val[u] = __ldg(bv);
            dst[u] = sv;
          }
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (dst[u] != nullptr) *dst[u] = val[u];
    }
  }
}

}  // namespace
}  // namespace saf

using namespace saf;

namespace {
int32_t ulysses_launch(bool pack, void* const* seq, int32_t T, int32_t dtype, int64_t B, int64_t s,
                       int64_t H, int64_t D, int64_t stride_b, int64_t stride_s, int64_t stride_h,
                       const int32_t* head_off, int32_t P, void* buf, void* stream) {
  if (seq == nullptr || buf == nullptr || head_off == nullptr) return SAF_ERR_ARG;
  if (T < 1 || T > kMaxTensors || P < 1 || P > kMaxPeers) return SAF_ERR_SHAPE;
  for (int t = 0; t < T; ++t)
    if (seq[t] == nullptr) return SAF_ERR_ARG;
  if (dtype != SAF_BF16 && dtype != SAF_F16 && dtype != SAF_F32) return SAF_ERR_DTYPE;
  const int64_t elem = dtype == SAF_F32 ? 4 : 2;
  if (B <= 0 || s < 0 || H <= 0 || D <= 0 || B > (1 << 20) || s > (1 << 30)) return SAF_ERR_SHAPE;
  if ((D * elem) % 16 != 0) return SAF_ERR_SHAPE;
  const int64_t v = 16 / elem;
  if (stride_b % v || stride_s % v || stride_h % v) return SAF_ERR_STRIDE;
  if ((reinterpret_cast<uintptr_t>(buf) & 15) != 0) return SAF_ERR_STRIDE;
  for (int t = 0; t < T; ++t)
    if ((reinterpret_cast<uintptr_t>(seq[t]) & 15) != 0) return SAF_ERR_STRIDE;
  if (head_off[0] != 0 || head_off[P] != H) return SAF_ERR_SHAPE;
  UlyssesParams p{};
  for (int t = 0; t < T; ++t) p.seq[t] = seq[t];
  p.buf = buf;
  p.s_b = stride_b;
  p.s_s = stride_s;
  p.s_h = stride_h;
  int hmax = 0;
  p.chunk_off[0] = 0;
  for (int j = 0; j < P; ++j) {
    const int hj = head_off[j + 1] - head_off[j];
    if (hj < 0) return SAF_ERR_SHAPE;
    hmax = hj > hmax ? hj : hmax;
    p.head_off[j] = head_off[j];
    p.chunk_off[j + 1] = p.chunk_off[j] + s * B * T * hj * D;
  }
  p.head_off[P] = head_off[P];
  p.T = T;
  p.B = static_cast<int32_t>(B);
  p.s = static_cast<int32_t>(s);
  p.D = static_cast<int32_t>(D);
  p.vec = static_cast<int32_t>(D * elem / 16);
  if (s == 0) return SAF_OK;
  int32_t rc;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(buf)) != SAF_OK) return rc;
  const int64_t inner = static_cast<int64_t>(T) * hmax * p.vec;  // vectors per row of the largest chunk
  if (inner == 0) return SAF_OK;
  if (s * B >= (int64_t(1) << 31) || inner >= (int64_t(1) << 31)) return SAF_ERR_SHAPE;
  // x: the vectors of one row (a warp multiple, at most 1024), y: rows per CTA
  const unsigned bx = static_cast<unsigned>(std::min<int64_t>(1024, (inner + 31) / 32 * 32));
  const unsigned by = std::max(1u, 256u / bx);
  const int64_t row_blocks = (s * B + by - 1) / by;
  dim3 block(bx, by);
  dim3 grid(static_cast<unsigned>(std::min<int64_t>(row_blocks, 148 * 16)), static_cast<unsigned>(P));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pack)
    ulysses_copy_kernel<true><<<grid, block, 0, st>>>(p);
  else
    ulysses_copy_kernel<false><<<grid, block, 0, st>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
}  // namespace

extern "C" int32_t saf_ulysses_pack(void* const* seq, int32_t T, int32_t dtype, int64_t B, int64_t s,
                                    int64_t H, int64_t D, int64_t stride_b, int64_t stride_s,
                                    int64_t stride_h, const int32_t* head_off, int32_t P, void* buf,
                                    void* stream) {
  return ulysses_launch(true, seq, T, dtype, B, s, H, D, stride_b, stride_s, stride_h, head_off, P, buf,
                        stream);
}

extern "C" int32_t saf_ulysses_unpack(const void* buf, int32_t T, int32_t dtype, int64_t B, int64_t s,
                                      int64_t H, int64_t D, int64_t stride_b, int64_t stride_s,
                                      int64_t stride_h, const int32_t* head_off, int32_t P,
                                      void* const* seq, void* stream) {
  return ulysses_launch(false, seq, T, dtype, B, s, H, D, stride_b, stride_s, stride_h, head_off, P,
                        const_cast<void*>(buf), stream);
}
