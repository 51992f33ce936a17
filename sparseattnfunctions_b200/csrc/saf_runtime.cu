// saf_runtime.cu -- library-wide runtime pieces: the per-device status word,
// the device-wait budget, tensor-map encoding and the small C entry points
// (version, status strings, device check, status read-back).
#include <atomic>
#include <mutex>

#include "saf_common.cuh"

namespace {

// Sticky status flags, one word per device (each device holds its own copy of
// a __device__ global).  Kernels receive its address as a parameter.
__device__ unsigned int g_saf_device_status = 0;

constexpr int kMaxDevices = 64;
unsigned int* g_status_ptr[kMaxDevices] = {nullptr};
std::mutex g_status_mu;

std::atomic<uint64_t> g_wait_budget_ns{1000000000ull};  // 1 s

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn g_encode = nullptr;
std::once_flag g_encode_once;

}  // namespace

namespace saf {

unsigned int* device_status_ptr() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_status_mu);
  if (g_status_ptr[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_saf_device_status) != cudaSuccess) return nullptr;
    g_status_ptr[dev] = static_cast<unsigned int*>(p);
  }
  return g_status_ptr[dev];
}

uint64_t wait_budget_ns() { return g_wait_budget_ns.load(); }

CUresult encode_tensor_map(CUtensorMap* map, CUtensorMapDataType dtype, cuuint32_t rank,
                           void* gaddr, const cuuint64_t* dims, const cuuint64_t* strides_bytes,
                           const cuuint32_t* box, CUtensorMapSwizzle swizzle) {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<EncodeTiledFn>(fn);
    }
  });
  if (g_encode == nullptr) return CUDA_ERROR_NOT_FOUND;
  cuuint32_t elem_strides[5] = {1, 1, 1, 1, 1};
  return g_encode(map, dtype, rank, gaddr, dims, strides_bytes, box, elem_strides,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

// Builds a 4-D tensor map over a [B,H,S,D] 16-bit tensor with a box of
// `rows` x 64 elements and 128-byte swizzle.
int32_t make_qkv_map(CUtensorMap* map, const saf_tensor4* t, int rows) {
  const uint64_t eb = 2;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(t->D), static_cast<cuuint64_t>(t->S),
                        static_cast<cuuint64_t>(t->H), static_cast<cuuint64_t>(t->B)};
  uint64_t sh = static_cast<uint64_t>(t->stride_h), sb = static_cast<uint64_t>(t->stride_b);
  // Extent-1 dims take any legal stride.
  if (t->H == 1) sh = static_cast<uint64_t>(t->stride_s) * t->S;
  if (t->B == 1) sb = sh * t->H;
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(t->stride_s) * eb, sh * eb, sb * eb};
  for (int i = 0; i < 3; ++i)
    if (strides[i] % 16 != 0 || strides[i] == 0 || strides[i] >= (1ull << 40))
      return SAF_ERR_STRIDE;
  cuuint32_t box[4] = {64u, static_cast<cuuint32_t>(rows), 1u, 1u};
  const CUtensorMapDataType dt =
      t->dtype == SAF_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = encode_tensor_map(map, dt, 4, t->data, dims, strides, box,
                                 CU_TENSOR_MAP_SWIZZLE_128B);
  return r == CUDA_SUCCESS ? SAF_OK : SAF_ERR_STRIDE;
}

bool current_device_is_sm100() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  int major = 0, minor = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess)
    return false;
  if (cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
    return false;
  return major == 10 && minor == 0;
}

int32_t DeviceScope::bind(const void* ptr) {
  cudaPointerAttributes attr;
  if (cudaPointerGetAttributes(&attr, ptr) != cudaSuccess) {
    cudaGetLastError();
    return SAF_ERR_ARG;
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) return SAF_ERR_ARG;
  int cur = -1;
  if (cudaGetDevice(&cur) != cudaSuccess) return SAF_ERR_CUDA;
  if (cur != attr.device) {
    if (cudaSetDevice(attr.device) != cudaSuccess) return SAF_ERR_CUDA;
    if (prev_ < 0) prev_ = cur;
  }
  return SAF_OK;
}

DeviceScope::~DeviceScope() {
  if (prev_ >= 0) cudaSetDevice(prev_);
}

namespace {
// Waits on an mbarrier that nothing ever arrives on: the bounded wait gives
// up after the budget and records SAF_DEV_TIMEOUT, as every kernel's waits do.
__global__ void selftest_timeout_kernel(unsigned int* status, uint64_t budget_ns) {
  __shared__ alignas(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait(smem_u32(&bar), 0, &abort_flag, status, budget_ns);
  __syncthreads();
}
}  // namespace
}  // namespace saf

extern "C" {

int32_t saf_abi_version(void) { return SAF_ABI_VERSION; }

const char* saf_status_string(int32_t s) {
  switch (s) {
    case SAF_OK: return "ok";
    case SAF_ERR_SHAPE: return "bad or unsupported shape";
    case SAF_ERR_DTYPE: return "bad or unsupported dtype";
    case SAF_ERR_STRIDE: return "bad stride or alignment";
    case SAF_ERR_CUDA: return "CUDA runtime error";
    case SAF_ERR_TIMEOUT: return "device wait timed out";
    case SAF_ERR_NCCL: return "collective error";
    case SAF_ERR_ARG: return "bad argument";
    case SAF_ERR_UNSUPPORTED: return "unsupported device or configuration";
    case SAF_ERR_WORKSPACE: return "workspace missing or too small";
    default: return "unknown status";
  }
}

int32_t saf_device_check(int32_t device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) return SAF_ERR_CUDA;
  if (device < 0 || device >= count) return SAF_ERR_ARG;
  int major = 0, minor = 0;
  SAF_CUDA_TRY(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  SAF_CUDA_TRY(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  return (major == 10 && minor == 0) ? SAF_OK : SAF_ERR_UNSUPPORTED;
}

void saf_set_wait_budget_ns(uint64_t ns) { g_wait_budget_ns.store(ns); }
uint64_t saf_get_wait_budget_ns(void) { return g_wait_budget_ns.load(); }

int32_t saf_selftest_timeout(uint64_t budget_ns, void* stream) {
  unsigned int* st = saf::device_status_ptr();
  if (st == nullptr) return SAF_ERR_CUDA;
  if (budget_ns > 10000000000ull) return SAF_ERR_ARG;  // at most 10 s
  saf::selftest_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(st, budget_ns);
  SAF_CUDA_TRY(cudaGetLastError());
  return SAF_OK;
}

int32_t saf_read_device_status(int32_t device, uint32_t* flags_out, int32_t clear) {
  if (flags_out == nullptr) return SAF_ERR_ARG;
  int prev = 0;
  SAF_CUDA_TRY(cudaGetDevice(&prev));
  SAF_CUDA_TRY(cudaSetDevice(device));
  int32_t rc = SAF_OK;
  unsigned int* p = saf::device_status_ptr();
  unsigned int v = 0;
  if (p == nullptr || cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&v, p, sizeof(v), cudaMemcpyDeviceToHost) != cudaSuccess) {
    rc = SAF_ERR_CUDA;
  } else {
    *flags_out = v;
    if (clear) {
      unsigned int zero = 0;
      if (cudaMemcpy(p, &zero, sizeof(zero), cudaMemcpyHostToDevice) != cudaSuccess)
        rc = SAF_ERR_CUDA;
    }
  }
  cudaSetDevice(prev);
  return rc;
}

}  // extern "C"
