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

// kPack: seq -> buf; otherwise buf -> seq.  One thread per 16-byte vector
// (consecutive lanes cover consecutive vectors of a row: coalesced on both
// sides), 32-bit index arithmetic.
template <bool kPack>
__global__ void __launch_bounds__(256) ulysses_copy_kernel(const UlyssesParams p) {
  const int j = blockIdx.y;
  const int hj = p.head_off[j + 1] - p.head_off[j];
  const int total = p.s * p.B * p.T * hj * p.vec;
  const int idx = static_cast<int>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  // chunk order: (s, b, t, h, vector)
  const int v = idx % p.vec;
  const int r = idx / p.vec;
  const int h = r % hj;
  const int q1 = r / hj;
  const int t = q1 % p.T;
  const int q2 = q1 / p.T;
  const int b = q2 % p.B;
  const int s = q2 / p.B;
  const int64_t elem_bytes = 16LL * p.vec / p.D;  // vec = D * element size / 16
  uint4* bufv = reinterpret_cast<uint4*>(static_cast<char*>(p.buf) + p.chunk_off[j] * elem_bytes) + idx;
  uint4* seqv = reinterpret_cast<uint4*>(static_cast<char*>(p.seq[t]) +
                                         (static_cast<int64_t>(b) * p.s_b + static_cast<int64_t>(s) * p.s_s +
                                          static_cast<int64_t>(p.head_off[j] + h) * p.s_h) * elem_bytes) + v;
  if constexpr (kPack) {
    *bufv = __ldg(seqv);
  } else {
    *seqv = __ldg(bufv);
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
  const int64_t most = s * B * T * static_cast<int64_t>(hmax) * p.vec;  // vectors of the largest chunk
  if (most == 0) return SAF_OK;
  if (most >= (int64_t(1) << 31)) return SAF_ERR_SHAPE;
  dim3 grid(static_cast<unsigned>((most + 255) / 256), static_cast<unsigned>(P));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pack)
    ulysses_copy_kernel<true><<<grid, 256, 0, st>>>(p);
  else
    ulysses_copy_kernel<false><<<grid, 256, 0, st>>>(p);
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
