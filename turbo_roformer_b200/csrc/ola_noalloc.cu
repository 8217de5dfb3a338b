// trc_ola_noalloc: the chunk overlap-add for callers that cannot allocate device memory.
//
// trc_ola stages the Hamming window and the chunk starts in buffers it obtains with cudaMalloc and
// cudaMallocAsync. Some callers cannot allow that: audio plugins whose host application owns all device
// memory through its own pool and forbids allocations of their own, or real-time audio hosts that must
// not take the allocator's locks on their processing thread. For them this entry point keeps the two
// staging arrays in fixed, file-scope device arrays of this library instead. They exist once per GPU
// context that loads the library and stay allocated until the process exits (8 MiB + 64 KiB each).
//
// Set-up: the first call in a CUDA context (the device's primary context, or a context the caller made
// current through the driver API) looks up the arrays' device addresses in that context; make that first
// call before any stream capture. The window array then keeps the window of the last chunk length
// uploaded in that context, so a call with the same chunk length as the previous one uploads only the
// starts (a copy of 8 bytes per chunk from pageable host memory). Every call shares the arrays, so calls
// that may overlap on the GPU race: the caller serialises them (one stream, or its own ordering).
#include <cuda.h>
#include <cuda_runtime.h>

#include <cmath>
#include <mutex>

#include "../../include/trcuda.h"
#include "internal.h"

namespace {

constexpr int64_t kMaxChunkSamples = TRC_OLA_NOALLOC_MAX_CHUNK;   // Hamming window length limit
constexpr int kMaxChunks = TRC_OLA_NOALLOC_MAX_CHUNKS;           // number of chunk starts limit
constexpr int kMaxContexts = 64;
constexpr int kHostBlock = 4096;  // window samples computed per host staging step

static __device__ __align__(256) float g_ola_window[kMaxChunkSamples];
static __device__ __align__(256) int64_t g_ola_starts[kMaxChunks];

// The arrays as seen from one CUDA context, and the chunk length whose window the array holds there.
struct ContextScratch {
  CUcontext ctx = nullptr;
  float* window = nullptr;
  int64_t* starts = nullptr;
  int64_t window_len = 0;  // 0: the window array holds no complete window
};

std::mutex g_scratch_mu;
ContextScratch g_scratch[kMaxContexts];
int g_n_scratch = 0;

using CtxGetCurrentFn = CUresult (*)(CUcontext*);

CtxGetCurrentFn ctx_get_current() {
  static CtxGetCurrentFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(p);
  }
  return fn;
}

// Looks up the calling thread's current context's record, creating it on the first call in that context:
// the arrays' host-side names are translated into device addresses with that context current. Host code
// must never pass the array names themselves to a kernel. Called with g_scratch_mu held.
cudaError_t scratch_for_current_context(ContextScratch** out) {
  void* w = nullptr;
  CtxGetCurrentFn get = ctx_get_current();
  if (!get) return cudaErrorNotSupported;
  CUcontext ctx = nullptr;
  if (get(&ctx) != CUDA_SUCCESS) return cudaErrorDeviceUninitialized;
  if (!ctx) {  // no context bound yet: the symbol lookup makes the runtime bind the device's primary one
    cudaError_t e = cudaGetSymbolAddress(&w, g_ola_window);
    if (e != cudaSuccess) return e;
    if (get(&ctx) != CUDA_SUCCESS || !ctx) return cudaErrorDeviceUninitialized;
  }
  for (int i = 0; i < g_n_scratch; ++i) {
    if (g_scratch[i].ctx == ctx) {
      *out = &g_scratch[i];
      return cudaSuccess;
    }
  }
  if (g_n_scratch == kMaxContexts) return cudaErrorLaunchOutOfResources;
  void* st = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&w, g_ola_window);
  if (e != cudaSuccess) return e;
  if ((e = cudaGetSymbolAddress(&st, g_ola_starts)) != cudaSuccess) return e;
  ContextScratch& s = g_scratch[g_n_scratch++];
  s.ctx = ctx;
  s.window = static_cast<float*>(w);
  s.starts = static_cast<int64_t*>(st);
  s.window_len = 0;
  *out = &s;
  return cudaSuccess;
}

}  // namespace

namespace trc {
int set_last_error(int code, const char* msg);  // api.cu
}

extern "C" int trc_ola_noalloc(const float* d_chunks, int64_t chunk_out_len, const int64_t* h_starts, int n_chunks,
                               int64_t chunk, int64_t n, float* d_result, void* stream) {
  if (!d_chunks || !h_starts || !d_result || n_chunks < 1 || chunk < 1 || n < 1 || chunk_out_len < 1 ||
      chunk_out_len > chunk)
    return trc::set_last_error(TRC_E_INVALID, "bad overlap-add arguments");
  if (chunk > kMaxChunkSamples)
    return trc::set_last_error(TRC_E_INVALID, "trc_ola_noalloc: chunk longer than TRC_OLA_NOALLOC_MAX_CHUNK samples");
  if (n_chunks > kMaxChunks)
    return trc::set_last_error(TRC_E_INVALID, "trc_ola_noalloc: more than TRC_OLA_NOALLOC_MAX_CHUNKS chunks");
  for (int i = 0; i < n_chunks; ++i) {
    if (h_starts[i] < 0 || h_starts[i] + chunk > n) return trc::set_last_error(TRC_E_INVALID, "chunk out of range");
    if (i && h_starts[i] <= h_starts[i - 1]) return trc::set_last_error(TRC_E_INVALID, "starts must be increasing");
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  ContextScratch* s = nullptr;
  if (scratch_for_current_context(&s) != cudaSuccess)
    return trc::set_last_error(TRC_E_CUDA, "cudaGetSymbolAddress failed for the overlap-add scratch");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Every value the kernel reads is written before it runs (the window when the chunk length changes,
  // the starts on every call), so nothing needs clearing. The window is computed in float64 and rounded
  // to float32 exactly like the allocating entry point, a block at a time through a stack buffer.
  if (s->window_len != chunk) {
    s->window_len = 0;
    float block[kHostBlock];
    for (int64_t k0 = 0; k0 < chunk; k0 += kHostBlock) {
      const int64_t m = chunk - k0 < kHostBlock ? chunk - k0 : kHostBlock;
      for (int64_t k = 0; k < m; ++k) {
        block[k] = chunk == 1 ? 1.0f
                              : (float)(0.54 - 0.46 * std::cos(2.0 * M_PI * (double)(k0 + k) / (double)(chunk - 1)));
      }
      // pageable source: the copy is staged before cudaMemcpyAsync returns, so `block` can be reused
      if (cudaMemcpyAsync(s->window + k0, block, sizeof(float) * m, cudaMemcpyHostToDevice, st) != cudaSuccess)
        return trc::set_last_error(TRC_E_CUDA, "window upload failed");
    }
    s->window_len = chunk;
  }
  if (cudaMemcpyAsync(s->starts, h_starts, sizeof(int64_t) * n_chunks, cudaMemcpyHostToDevice, st) != cudaSuccess)
    return trc::set_last_error(TRC_E_CUDA, "starts upload failed");
  trc::launch_chunk_ola(d_chunks, chunk_out_len, s->starts, n_chunks, s->window, n, d_result, st);
  trc::count_launches(1);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return trc::set_last_error(TRC_E_CUDA, cudaGetErrorString(e));
  return TRC_OK;
}
