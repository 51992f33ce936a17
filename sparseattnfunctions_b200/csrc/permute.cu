// Token permutation / padding of [B, H, S, D] tensors: out[g, s, :] =
// x[g, perm[s], :] for s < S_out (perm[s] == -1 writes a zero row), for the
// heads g = b*H + h listed in `heads` (all heads when null).
//
// SmartAttention runs the heads it classifies as "temporal" on the video
// tokens reordered from (t, h, w) to (h, w, t) order and reorders their
// output back (SmartAttention.py:16-27 process / process_back).  With both
// directions expressed as one gather by a token permutation, this is a
// single HBM pass per tensor; the head list lets the inverse permutation
// write only the heads that took the reordered path.  SildingTileAttention
// uses the padding form to place every 117-token tile in its own 128-row
// block (and the inverse to read the output back).
//
// One thread per 16-byte vector of a D row (D * element size a multiple of
// 16 bytes and 16-byte aligned rows, host-checked), else one per element.
#include <cstdint>

#include "saf_common.cuh"

namespace saf {
namespace {

struct PermuteParams {
  const void* x;
  void* out;
  int64_t x_sb, x_sh, x_ss, o_sb, o_sh, o_ss;  // in units (16-byte vectors or elements)
  const int32_t* perm;
  const int32_t* heads;
  int H, S_in, S_out, units;  // units per D row
  int64_t groups_total;  // B * H (bound of the head list)
  unsigned int* status;
};

template <typename U>
__global__ void __launch_bounds__(256) permute_tokens_kernel(const PermuteParams p) {
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<int64_t>(p.S_out) * p.units) return;
  const int s = static_cast<int>(idx / p.units), u = static_cast<int>(idx - static_cast<int64_t>(s) * p.units);
  const int g = p.heads ? p.heads[blockIdx.y] : static_cast<int>(blockIdx.y);
  const int src = p.perm[s];
  if (g < 0 || g >= p.groups_total || src < -1 || src >= p.S_in) {  // bad index: flag, skip the copy
    atomicOr(p.status, SAF_DEV_BADINDEX);
    return;
  }
  const int b = g / p.H, h = g % p.H;
  U* os = static_cast<U*>(p.out) + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(s) * p.o_ss + u;
  if (src < 0) {  // padding row
    *os = U{};
    return;
  }
  const U* xs = static_cast<const U*>(p.x) + b * p.x_sb + h * p.x_sh + static_cast<int64_t>(src) * p.x_ss + u;
  *os = __ldg(xs);
}

}  // namespace
}  // namespace saf

using namespace saf;

extern "C" int32_t saf_permute_tokens(const void* x, void* out, int32_t dtype, int64_t B, int64_t H,
                                      int64_t S, int64_t S_out, int64_t D, int64_t x_sb, int64_t x_sh,
                                      int64_t x_ss,
                                      int64_t o_sb, int64_t o_sh, int64_t o_ss, const int32_t* perm,
                                      const int32_t* heads, int64_t n_heads, void* stream) {
  if (x == nullptr || out == nullptr || perm == nullptr) return SAF_ERR_ARG;
  if (dtype != SAF_BF16 && dtype != SAF_F16 && dtype != SAF_F32) return SAF_ERR_DTYPE;
  if (B <= 0 || H <= 0 || S <= 0 || S_out <= 0 || D <= 0 || S > (1 << 30) || S_out > (1 << 30) ||
      D > (1 << 16))
    return SAF_ERR_SHAPE;
  const int64_t groups = heads ? n_heads : B * H;
  if (groups < 0 || groups > 65535) return SAF_ERR_SHAPE;
  if (groups == 0) return SAF_OK;
  const int64_t elem = dtype == SAF_F32 ? 4 : 2;
  const int64_t v = 16 / elem;
  const bool vec = (D * elem) % 16 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
                   (reinterpret_cast<uintptr_t>(out) & 15) == 0 && x_sb % v == 0 && x_sh % v == 0 &&
                   x_ss % v == 0 && o_sb % v == 0 && o_sh % v == 0 && o_ss % v == 0;
  int32_t rc;
  DeviceScope dev_scope;
  if ((rc = dev_scope.bind(x)) != SAF_OK) return rc;
  const int64_t div = vec ? v : 1;
  PermuteParams p{x, out, x_sb / div, x_sh / div, x_ss / div, o_sb / div, o_sh / div, o_ss / div,
                  perm, heads, static_cast<int>(H), static_cast<int>(S), static_cast<int>(S_out),
                  static_cast<int>(D / div),
                  B * H, device_status_ptr()};
  if (p.status == nullptr) return SAF_ERR_CUDA;
  const int64_t total = S_out * p.units;
  dim3 grid(static_cast<unsigned>((total + 255) / 256), static_cast<unsigned>(groups));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (vec)
    permute_tokens_kernel<uint4><<<grid, 256, 0, st>>>(p);
  else if (elem == 4)
    permute_tokens_kernel<uint32_t><<<grid, 256, 0, st>>>(p);
  else
    permute_tokens_kernel<uint16_t><<<grid, 256, 0, st>>>(p);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}
