// Runtime entry points: thread-local error messages, device selection, the flat-buffer
// allocator primitives and the dtype cast kernel.
#include <cstdarg>
#include <cstdio>
#include <cstring>

#include "nt_common.cuh"

namespace nt {

static thread_local char g_last_error[512] = "";

void set_error(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
}

int cuda_fail(cudaError_t err, const char* what) {
  set_error("%s: %s (%s)", what, cudaGetErrorString(err), cudaGetErrorName(err));
  return err == cudaErrorMemoryAllocation ? NT_ENOMEM : NT_ECUDA;
}

static int g_sm_count[64] = {0};

int current_sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
    g_sm_count[dev] = n;
  }
  return g_sm_count[dev];
}

// Conversion kernel: 8 elements per thread on aligned storage, scalar otherwise.
template <int SRC, int DST>
__global__ void cast_kernel(void* dst, const void* src, int64_t count, int vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (vec) {
    const int64_t nvec = count / 8;
    for (int64_t i = t; i < nvec; i += stride) {
      float v[8];
      load8<SRC>(src, i * 8, v);
      store8<DST>(dst, i * 8, v);
    }
    for (int64_t i = nvec * 8 + t; i < count; i += stride) store1<DST>(dst, i, load1<SRC>(src, i));
  } else {
    for (int64_t i = t; i < count; i += stride) store1<DST>(dst, i, load1<SRC>(src, i));
  }
}

template <int SRC, int DST>
static int launch_cast(void* dst, const void* src, int64_t count, cudaStream_t stream) {
  const int vec = aligned16(dst) && aligned16(src);
  int64_t work = vec ? (count + 7) / 8 : count;
  int64_t blocks = (work + 255) / 256;
  const int64_t cap = (int64_t)current_sm_count() * 8;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  cast_kernel<SRC, DST><<<(unsigned)blocks, 256, 0, stream>>>(dst, src, count, vec);
  return launch_status("nt_cast launch");
}

}  // namespace nt

using namespace nt;

extern "C" {

int nt_abi_version(void) { return NT_ABI_VERSION; }

const char* nt_last_error(void) { return g_last_error; }

int nt_device_init(int device) {
  int count = 0;
  cudaError_t err = cudaGetDeviceCount(&count);
  if (err != cudaSuccess) return cuda_fail(err, "cudaGetDeviceCount");
  if (device < 0 || device >= count) {
    set_error("device %d is out of range (found %d CUDA devices)", device, count);
    return NT_EINVAL;
  }
  err = cudaSetDevice(device);
  if (err != cudaSuccess) return cuda_fail(err, "cudaSetDevice");
  (void)current_sm_count();
  return NT_OK;
}

int nt_sm_count(int* count) {
  if (!count) { set_error("nt_sm_count: count is NULL"); return NT_EINVAL; }
  *count = current_sm_count();
  return NT_OK;
}

int nt_malloc(void** ptr, size_t bytes) {
  if (!ptr) { set_error("nt_malloc: ptr is NULL"); return NT_EINVAL; }
  *ptr = nullptr;
  if (bytes == 0) return NT_OK;
  cudaError_t err = cudaMalloc(ptr, bytes);
  if (err != cudaSuccess) {
    cudaGetLastError();
    size_t free_b = 0, total_b = 0;
    cudaMemGetInfo(&free_b, &total_b);
    int dev = -1;
    cudaGetDevice(&dev);
    set_error("out of memory on cuda:%d: requested=%zu bytes, free=%zu bytes, total=%zu bytes",
              dev, bytes, free_b, total_b);
    return NT_ENOMEM;
  }
  return NT_OK;
}

int nt_free(void* ptr) {
  if (!ptr) return NT_OK;
  cudaError_t err = cudaFree(ptr);
  if (err != cudaSuccess) return cuda_fail(err, "cudaFree");
  return NT_OK;
}

int nt_mem_info(size_t* free_bytes, size_t* total_bytes) {
  if (!free_bytes || !total_bytes) { set_error("nt_mem_info: NULL output"); return NT_EINVAL; }
  cudaError_t err = cudaMemGetInfo(free_bytes, total_bytes);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemGetInfo");
  return NT_OK;
}

int nt_memset_async(void* ptr, int value, size_t bytes, void* stream) {
  if (bytes == 0) return NT_OK;
  if (!ptr) { set_error("nt_memset_async: ptr is NULL"); return NT_EINVAL; }
  cudaError_t err = cudaMemsetAsync(ptr, value, bytes, as_stream(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemsetAsync");
  return NT_OK;
}

int nt_memcpy_async(void* dst, const void* src, size_t bytes, void* stream) {
  if (bytes == 0) return NT_OK;
  if (!dst || !src) { set_error("nt_memcpy_async: NULL pointer"); return NT_EINVAL; }
  cudaError_t err = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, as_stream(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpyAsync");
  return NT_OK;
}

int nt_memcpy_sync(void* dst, const void* src, size_t bytes) {
  if (bytes == 0) return NT_OK;
  if (!dst || !src) { set_error("nt_memcpy_sync: NULL pointer"); return NT_EINVAL; }
  cudaError_t err = cudaMemcpy(dst, src, bytes, cudaMemcpyDefault);
  if (err != cudaSuccess) return cuda_fail(err, "cudaMemcpy");
  return NT_OK;
}

int nt_stream_synchronize(void* stream) {
  cudaError_t err = cudaStreamSynchronize(as_stream(stream));
  if (err != cudaSuccess) return cuda_fail(err, "cudaStreamSynchronize");
  return NT_OK;
}

int nt_cast(void* dst, int dst_dtype, const void* src, int src_dtype, int64_t count, void* stream) {
  nt::TraceRange trace("nt_cast");
  if (count < 0) { set_error("nt_cast: negative count"); return NT_EINVAL; }
  if (count == 0) return NT_OK;
  if (!dst || !src) { set_error("nt_cast: NULL pointer"); return NT_EINVAL; }
  if (dtype_size(dst_dtype) == 0 || dtype_size(src_dtype) == 0) {
    set_error("nt_cast: unsupported dtype pair (%d -> %d)", src_dtype, dst_dtype);
    return NT_EUNSUPPORTED;
  }
  cudaStream_t s = as_stream(stream);
#define NT_CAST_CASE(S, D) \
  if (src_dtype == S && dst_dtype == D) return launch_cast<S, D>(dst, src, count, s);
  NT_CAST_CASE(NT_F32, NT_F32) NT_CAST_CASE(NT_F32, NT_F16) NT_CAST_CASE(NT_F32, NT_BF16)
  NT_CAST_CASE(NT_F16, NT_F32) NT_CAST_CASE(NT_F16, NT_F16) NT_CAST_CASE(NT_F16, NT_BF16)
  NT_CAST_CASE(NT_BF16, NT_F32) NT_CAST_CASE(NT_BF16, NT_F16) NT_CAST_CASE(NT_BF16, NT_BF16)
#undef NT_CAST_CASE
  set_error("nt_cast: unsupported dtype pair");
  return NT_EUNSUPPORTED;
}

}  // extern "C"
