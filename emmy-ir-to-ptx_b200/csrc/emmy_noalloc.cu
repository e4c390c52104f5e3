// emmy_noalloc.cu -- an f32 sum that allocates nothing (emmy_rt_sum_f32_noalloc).
//
// Some hosts that bind this library may not allocate device memory when they call
// it: a service whose memory pool has already reserved the device's HBM (so a
// stray cudaMalloc fails or fragments the pool), or a latency-critical loop in
// which a cudaFree would synchronise the whole device. The full-sum kernel that
// compile.py emits needs a few KB of scratch for its cross-CTA finish; in the
// PTX path the driver reserves that scratch when the module is loaded. This
// file offers the same reduction with its scratch in a fixed, file-scope
// device array, so a call needs only the caller's input and output buffers.
//
// Limits and sharing rules:
//  * At most EMMY_RT_NOALLOC_MAX_CTAS (4096) CTAs; larger grids are rejected.
//    The array is (4096 + 64) * 4 bytes = 16,640 bytes, and every GPU that
//    loads this library keeps that much until the process exits.
//  * Every call on a device uses the same array. Two calls that overlap on the
//    GPU (different streams, or different host threads) race on it and give
//    wrong results; serialise them.
//  * The first call on each device looks up the array's device address with
//    cudaGetSymbolAddress (with that device current). Under CUDA's lazy module
//    loading (the default since CUDA 12.2) that first call is also what loads
//    this file's device code and its 16,640-byte array onto the device, so make
//    it before the host's pool reserves the device's memory, and before any
//    stream capture begins.
//  * Calls outside stream capture look the address up again (cheap once the
//    module is loaded), so a reset of the device's primary context (after
//    cudaDeviceReset, say) is picked up; a call on a capturing stream uses the
//    address of the last call made outside capture on that device.
//  * x and out must be 4-byte aligned (they are float arrays); other pointers
//    are refused before anything is launched.

#include "emmy_rt.h"

#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

// shared with emmy_rt.cpp: stores the message emmy_rt_last_error() returns
void emmy_rt_internal_set_error(const char *msg);

namespace {

constexpr int kThreads = 256;
constexpr int kMaxDevices = 64;
constexpr int kTicketSlot = EMMY_RT_NOALLOC_MAX_CTAS;   // uint32 index of the ticket

// partial sums (float bits) in [0, MAX_CTAS); the ticket counter at [MAX_CTAS]
static __device__ __align__(256) unsigned int emmy_noalloc_scratch[EMMY_RT_NOALLOC_MAX_CTAS + 64];

std::mutex g_mu;
unsigned int *g_scratch_addr[kMaxDevices] = {};


__device__ __forceinline__ float warp_sum(float v) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Block-wide sum; the result is valid in thread 0.
__device__ __forceinline__ float block_sum(float v, float *red) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  v = (threadIdx.x < kThreads / 32) ? red[threadIdx.x] : 0.f;
  if (warp == 0) v = warp_sum(v);
  return v;
}

__global__ void __launch_bounds__(kThreads)
sum_f32_noalloc_kernel(const float *__restrict__ x, unsigned long long n, float *out,
                       unsigned int *scratch) {
  __shared__ float red[kThreads / 32];
  __shared__ unsigned int last;
  const unsigned long long nthr = (unsigned long long)gridDim.x * kThreads;
  const unsigned long long gtid = (unsigned long long)blockIdx.x * kThreads + threadIdx.x;
  float acc = 0.f;
  unsigned long long start = gtid;
  if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
    const float4 *x4 = reinterpret_cast<const float4 *>(x);
    const unsigned long long nv = n / 4;
    for (unsigned long long c = gtid; c < nv; c += nthr) {
      float4 v = __ldg(x4 + c);
      acc += v.x;
      acc += v.y;
      acc += v.z;
      acc += v.w;
    }
    start = nv * 4 + gtid;
  }
  for (unsigned long long e = start; e < n; e += nthr) acc += __ldg(x + e);

  float part = block_sum(acc, red);
  if (threadIdx.x == 0) {
    scratch[blockIdx.x] = __float_as_uint(part);
    __threadfence();
    // wraps back to zero after the last CTA, so the counter is ready for the next call
    const unsigned int ticket = atomicInc(&scratch[kTicketSlot], gridDim.x - 1);
    last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  float t = 0.f;
  for (unsigned int i = threadIdx.x; i < gridDim.x; i += kThreads)
    t += __uint_as_float(__ldcg(&scratch[i]));
  __syncthreads();
  t = block_sum(t, red);
  if (threadIdx.x == 0) out[0] = t;
}

int fail(int code, const char *what, cudaError_t e) {
  char msg[512];
  snprintf(msg, sizeof(msg), "%s%s%s", what, e == cudaSuccess ? "" : ": ",
           e == cudaSuccess ? "" : cudaGetErrorString(e));
  emmy_rt_internal_set_error(msg);
  return code;
}

// Device address of the scratch array for the current device. Outside stream capture it is
// looked up on every call (so a context that was reset and made again is seen); a capturing
// stream uses the address the last uncaptured call on this device found, since a lookup that
// has to load the module is not allowed while a capture is running.
int scratch_for_current_device(cudaStream_t s, unsigned int **out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(EMMY_RT_ECUDA, "cudaGetDevice", e);
  if (dev < 0 || dev >= kMaxDevices) return fail(EMMY_RT_EINVAL, "device index out of range",
                                                  cudaSuccess);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(s, &cs);
  if (e != cudaSuccess) return fail(EMMY_RT_ECUDA, "cudaStreamIsCapturing", e);
  std::lock_guard<std::mutex> lock(g_mu);
  if (cs == cudaStreamCaptureStatusNone) {
    void *p = nullptr;
    e = cudaGetSymbolAddress(&p, emmy_noalloc_scratch);
    if (e != cudaSuccess) return fail(EMMY_RT_ECUDA, "cudaGetSymbolAddress", e);
    g_scratch_addr[dev] = static_cast<unsigned int *>(p);
  } else if (!g_scratch_addr[dev]) {
    return fail(EMMY_RT_EINVAL,
                "first call on this device made during stream capture: call once before "
                "capturing so the scratch address is known", cudaSuccess);
  }
  *out = g_scratch_addr[dev];
  return EMMY_RT_OK;
}

}  // namespace

extern "C" int emmy_rt_sum_f32_noalloc(uint64_t x, uint64_t n, uint64_t out, uint32_t grid,
                                       uint64_t stream) {
  if (!x || !out) return fail(EMMY_RT_EINVAL, "null buffer", cudaSuccess);
  if ((x | out) & 3u)
    return fail(EMMY_RT_EINVAL, "x and out must be 4-byte aligned (f32 arrays)", cudaSuccess);
  if (grid == 0 || grid > EMMY_RT_NOALLOC_MAX_CTAS) {
    char msg[160];
    snprintf(msg, sizeof(msg), "grid %u outside 1..%d (the fixed scratch holds %d partials)",
             grid, EMMY_RT_NOALLOC_MAX_CTAS, EMMY_RT_NOALLOC_MAX_CTAS);
    emmy_rt_internal_set_error(msg);
    return EMMY_RT_EINVAL;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(static_cast<uintptr_t>(stream));
  unsigned int *scratch = nullptr;
  int rc = scratch_for_current_device(s, &scratch);
  if (rc) return rc;
  // the ticket must start at zero even if an earlier call was cut short
  cudaError_t e = cudaMemsetAsync(scratch + kTicketSlot, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess) return fail(EMMY_RT_ECUDA, "cudaMemsetAsync", e);
  sum_f32_noalloc_kernel<<<grid, kThreads, 0, s>>>(
      reinterpret_cast<const float *>(static_cast<uintptr_t>(x)), n,
      reinterpret_cast<float *>(static_cast<uintptr_t>(out)), scratch);
  e = cudaGetLastError();
  if (e != cudaSuccess) return fail(EMMY_RT_ECUDA, "kernel launch", e);
  return EMMY_RT_OK;
}
