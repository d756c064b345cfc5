// emmy_sum_f32_noalloc -- a full-array f32 sum that allocates no memory.
//
// Why it exists: some callers of this library cannot call cudaMalloc at the
// point where they need a reduction -- plugin hosts whose enqueue callback
// must not allocate (the host framework owns all device memory through its
// own pool), and latency-critical loops where cudaMalloc's implicit
// device-wide synchronisation would stall every other stream.  The regular
// path (the compiled IR kernel of the full-reduction family) keeps its
// per-CTA partials in module scratch that the driver allocates when the PTX
// module is loaded.  This variant needs no module load and no allocation:
// its scratch is the file-scope array below, which every GPU that loads
// libemmyrt.so holds until the process exits.
//
// Limits and sharing rules:
//   - scratch: NOALLOC_SLOTS (1024) per-CTA partial sums plus one ticket
//     word, 4.25 KiB per device; the grid is clamped to NOALLOC_SLOTS CTAs,
//     so the scratch can never overflow;
//   - n: at most NOALLOC_MAX_ELEMS (2^31 - 1) elements (32-bit indexing);
//     larger n is rejected with EMMY_EINVAL and a message;
//   - every call on a device shares the one array and it keeps the previous
//     call's contents, so each call clears the ticket word (stream-ordered
//     cudaMemsetAsync) before its kernel; calls that overlap on the GPU
//     (for example on two streams at once) race on the scratch and must be
//     serialised by the caller;
//   - the first call in each CUDA context performs the set-up: with that
//     context's device current it resolves the device address of the array
//     with cudaGetSymbolAddress (checked) and caches it under the context
//     (the runtime's primary context, or a context the caller created with
//     the driver API and made current); make that first call before any
//     stream capture.  The cache is not refreshed after cudaDeviceReset (a
//     new primary context may reuse the old handle): a process that resets
//     a device must not call this entry point afterwards;
//   - failures of CUDA runtime calls return EMMY_ECUDART, with the runtime's
//     own message in emmy_last_error().
#include <cuda.h>  // CUcontext and the cuCtxGetCurrent signature only (no libcuda link)
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "emmyrt.h"

// Sets the thread-local message emmy_last_error() returns (emmyrt.cpp; not
// exported from the library).
void emmyrt_set_last_error(const char *msg);

namespace {

constexpr int NOALLOC_SLOTS = 1024;           // per-CTA partials
constexpr int NOALLOC_TICKET_WORD = 0;        // word 0: arrival ticket
constexpr int NOALLOC_PARTIAL_WORD = 64;      // partials start on their own 256-byte line
constexpr int NOALLOC_WORDS = NOALLOC_PARTIAL_WORD + NOALLOC_SLOTS;
constexpr size_t NOALLOC_MAX_ELEMS = 0x7fffffffu;
constexpr int NOALLOC_THREADS = 512;
constexpr int NOALLOC_MAX_CONTEXTS = 64;

// The only memory this entry point uses beyond the caller's buffers.
static __device__ __align__(256) unsigned int g_noalloc_scratch[NOALLOC_WORDS];

// The array's device address per CUDA context: each context that loads this
// library's kernels holds its own copy of the array.
struct ScratchEntry {
  CUcontext ctx;
  unsigned int *addr;
};
std::mutex g_setup_mu;
ScratchEntry g_scratch[NOALLOC_MAX_CONTEXTS] = {};
int g_scratch_used = 0;

__device__ __forceinline__ float warp_sum(float v) {
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  return v;
}

// Block-wide sum; every thread receives the result.
__device__ float block_sum(float v, float *slots) {
  v = warp_sum(v);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) slots[warp] = v;
  __syncthreads();
  const int nwarps = (blockDim.x + 31) >> 5;
  v = lane < nwarps ? slots[lane] : 0.0f;
  v = warp_sum(v);
  __syncthreads();  // slots may be reused by the caller
  return v;
}

__global__ void __launch_bounds__(NOALLOC_THREADS)
sum_noalloc_kernel(const float *__restrict__ x, uint32_t n, float *__restrict__ out,
                   unsigned int *scratch) {
  __shared__ float slots[32];
  __shared__ unsigned int is_last;
  float acc = 0.0f;
  const uint32_t tid = blockIdx.x * blockDim.x + threadIdx.x;
  const uint32_t stride = gridDim.x * blockDim.x;
  const uint32_t nvec = n / 4;
  const float4 *x4 = reinterpret_cast<const float4 *>(x);
  uint32_t i = tid;
  // four 16-byte loads in flight per thread, then the remainder
  for (; i + 3 * stride < nvec; i += 4 * stride) {
    float4 a = __ldcs(x4 + i), b = __ldcs(x4 + i + stride);
    float4 c = __ldcs(x4 + i + 2 * stride), d = __ldcs(x4 + i + 3 * stride);
    acc += ((a.x + a.y) + (a.z + a.w)) + ((b.x + b.y) + (b.z + b.w));
    acc += ((c.x + c.y) + (c.z + c.w)) + ((d.x + d.y) + (d.z + d.w));
  }
  for (; i < nvec; i += stride) {
    float4 a = __ldcs(x4 + i);
    acc += (a.x + a.y) + (a.z + a.w);
  }
  for (uint32_t j = nvec * 4 + tid; j < n; j += stride) acc += x[j];
  acc = block_sum(acc, slots);

  float *partials = reinterpret_cast<float *>(scratch + NOALLOC_PARTIAL_WORD);
  if (threadIdx.x == 0) {
    partials[blockIdx.x] = acc;
    __threadfence();
    const unsigned int ticket = atomicAdd(scratch + NOALLOC_TICKET_WORD, 1u);
    is_last = (ticket == gridDim.x - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  // The last CTA folds the partials in a fixed order, so the result does not
  // depend on which CTA finished last.
  float total = 0.0f;
  for (uint32_t j = threadIdx.x; j < gridDim.x; j += blockDim.x) total += __ldcg(partials + j);
  total = block_sum(total, slots);
  if (threadIdx.x == 0) {
    *out = total;
    scratch[NOALLOC_TICKET_WORD] = 0u;  // leave the ticket clear for the next call
  }
}

int set_error(int code, const char *msg) {
  char buf[256];
  snprintf(buf, sizeof buf, "emmy_sum_f32_noalloc: %s", msg);
  emmyrt_set_last_error(buf);
  return code;
}

int runtime_error(cudaError_t e) { return set_error(EMMY_ECUDART, cudaGetErrorString(e)); }

// The context current on this thread, through the runtime's driver entry
// point (the library does not link libcuda).
int current_context(CUcontext *ctx) {
  static CUresult (*get_current)(CUcontext *) = nullptr;
  if (get_current == nullptr) {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &fn, 12000,
                                                     cudaEnableDefault, &q);
    if (e != cudaSuccess) return runtime_error(e);
    if (q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(EMMY_ECUDART, "cuCtxGetCurrent is not available from the driver");
    get_current = reinterpret_cast<CUresult (*)(CUcontext *)>(fn);
  }
  *ctx = nullptr;
  if (get_current(ctx) != CUDA_SUCCESS)
    return set_error(EMMY_ECUDART, "cuCtxGetCurrent failed");
  return EMMY_OK;
}

// Device address of the scratch array in the current context (set-up on the
// first call in each context).
int scratch_for_current_context(unsigned int **out) {
  std::lock_guard<std::mutex> lock(g_setup_mu);
  CUcontext ctx = nullptr;
  int rc = current_context(&ctx);
  if (rc != EMMY_OK) return rc;
  for (int i = 0; ctx != nullptr && i < g_scratch_used; ++i) {
    if (g_scratch[i].ctx == ctx) {
      *out = g_scratch[i].addr;
      return EMMY_OK;
    }
  }
  // Set-up: resolve the array in the current context.  With no context
  // current, the runtime makes the current device's primary context current
  // here, and the entry is kept under that context.
  void *p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return runtime_error(e);
  if (ctx == nullptr) {
    rc = current_context(&ctx);
    if (rc != EMMY_OK) return rc;
  }
  if (ctx != nullptr && g_scratch_used < NOALLOC_MAX_CONTEXTS)
    g_scratch[g_scratch_used++] = ScratchEntry{ctx, static_cast<unsigned int *>(p)};
  *out = static_cast<unsigned int *>(p);
  return EMMY_OK;
}

}  // namespace

extern "C" int emmy_sum_f32_noalloc(emmy_dptr x, size_t n, emmy_dptr out, emmy_stream stream) {
  if (x == 0 || out == 0) return set_error(EMMY_EINVAL, "null buffer");
  if (n == 0 || n > NOALLOC_MAX_ELEMS)
    return set_error(EMMY_EINVAL, "n must be between 1 and 2^31 - 1 elements");
  if (x % 16 != 0) return set_error(EMMY_EINVAL, "x must be 16-byte aligned");
  if (out % 4 != 0) return set_error(EMMY_EINVAL, "out must be 4-byte aligned");
  unsigned int *scratch = nullptr;
  int rc = scratch_for_current_context(&scratch);
  if (rc != EMMY_OK) return rc;
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return runtime_error(e);
  const size_t nvec = (n + 3) / 4;
  size_t grid = (nvec + NOALLOC_THREADS * 8 - 1) / (NOALLOC_THREADS * 8);
  if (grid > size_t(sms) * 4) grid = size_t(sms) * 4;
  if (grid > size_t(NOALLOC_SLOTS)) grid = NOALLOC_SLOTS;
  if (grid < 1) grid = 1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // the ticket must start at zero; the partials are overwritten before use
  e = cudaMemsetAsync(scratch + NOALLOC_TICKET_WORD, 0, sizeof(unsigned int), s);
  if (e != cudaSuccess) return runtime_error(e);
  sum_noalloc_kernel<<<unsigned(grid), NOALLOC_THREADS, 0, s>>>(
      reinterpret_cast<const float *>(x), uint32_t(n), reinterpret_cast<float *>(out), scratch);
  e = cudaGetLastError();
  if (e != cudaSuccess) return runtime_error(e);
  return EMMY_OK;
}
