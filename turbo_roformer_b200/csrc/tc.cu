// Instantiation and launch of the tensor-core kernels (tcgen05 GEMM with fused epilogues, attention).
#include <atomic>

#include "attention.cuh"
#include "attention_time.cuh"
#include "gemm.cuh"
#include "internal.h"
#include "mlp.cuh"

namespace trc {

namespace {

// The dynamic shared-memory opt-in is per function and per device: set it once for each pair.
// `done` must be a distinct object per kernel instantiation (callers pass a function-local static).
template <typename Kern>
cudaError_t allow_smem(Kern kern, int bytes, std::atomic<unsigned long long>& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_relaxed) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit);
  return e;
}

constexpr int kBN = 256;
constexpr int kStages = 3;

template <int EPI, typename T>
cudaError_t launch_gemm_t(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap* mo, const GemmArgs& args,
                          int num_sms, cudaStream_t st) {
  // qkv: resident A tile (or streamed A, EPI_QKVS) + rotary rows take the space
  constexpr int kSt = is_qkv(EPI) ? 2 : kStages;
  using S = GemmSmem<kBN, kSt, EPI>;
  auto kern = gemm_kernel<kBN, kSt, EPI, T>;
  static std::atomic<unsigned long long> done{0};  // one per <EPI, T> instantiation
  cudaError_t e = allow_smem(kern, S::kBytes, done);
  if (e != cudaSuccess) return e;
  if (args.num_tiles <= 0) return cudaSuccess;
  const int grid = args.num_tiles < num_sms ? args.num_tiles : num_sms;
  kern<<<grid, kGemmThreads, S::kBytes, st>>>(ma, mb, mo[0], mo[1], mo[2], args);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_gemm_p(int epi, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap* mo,
                          const GemmArgs& args, int num_sms, cudaStream_t st) {
  switch (epi) {
    case EPI_QKV: return launch_gemm_t<EPI_QKV, T>(ma, mb, mo, args, num_sms, st);
    case EPI_RESNORM: return launch_gemm_t<EPI_RESNORM, T>(ma, mb, mo, args, num_sms, st);
    case EPI_GELU: return launch_gemm_t<EPI_GELU, T>(ma, mb, mo, args, num_sms, st);
    case EPI_MASK_TANH: return launch_gemm_t<EPI_MASK_TANH, T>(ma, mb, mo, args, num_sms, st);
    case EPI_MASK_GLU: return launch_gemm_t<EPI_MASK_GLU, T>(ma, mb, mo, args, num_sms, st);
    case EPI_BAND: return launch_gemm_t<EPI_BAND, T>(ma, mb, mo, args, num_sms, st);
    case EPI_F32: return launch_gemm_t<EPI_F32, T>(ma, mb, mo, args, num_sms, st);
    case EPI_QKVS: return launch_gemm_t<EPI_QKVS, T>(ma, mb, mo, args, num_sms, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
cudaError_t launch_attention_freq(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                                  const AttnArgs& args, int num_sms, cudaStream_t st) {
  auto kern = attention_freq_kernel<T>;
  static std::atomic<unsigned long long> done{0};  // one per <T> instantiation
  cudaError_t e = allow_smem(kern, AttnSmem::kBytes, done);
  if (e != cudaSuccess) return e;
  if (args.num_items <= 0) return cudaSuccess;
  const int grid = args.num_items < num_sms ? args.num_items : num_sms;
  kern<<<grid, kAttnThreads, AttnSmem::kBytes, st>>>(mq, mk, mv, args);
  return cudaGetLastError();
}

// Time mode: three query tiles per CTA (attention_time.cuh). The kernel moves registers between its
// warpgroups (setmaxnreg): the split must fit in what the launch gives the block, or the softmax warps'
// increase would never be granted.
template <typename T>
cudaError_t launch_attention_time(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                                  const AttnArgs& args, int num_sms, cudaStream_t st) {
  auto kern = attention_time_kernel<T>;
  static std::atomic<unsigned long long> done{0};
  cudaError_t e = allow_smem(kern, TaSmem::kBytes, done);
  if (e != cudaSuccess) return e;
  static std::atomic<int> regs{0};
  if (regs.load() == 0) {
    cudaFuncAttributes fa;
    if ((e = cudaFuncGetAttributes(&fa, kern)) != cudaSuccess) return e;
    regs.store(fa.numRegs);
  }
  if (4 * 32 * kTaRegsLow + 12 * 32 * kTaRegsHigh > kTaThreads * regs.load()) return cudaErrorInvalidConfiguration;
  if (args.num_items <= 0) return cudaSuccess;
  const int grid = args.num_items < num_sms ? args.num_items : num_sms;
  kern<<<grid, kTaThreads, TaSmem::kBytes, st>>>(mq, mk, mv, args);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_attention_t(const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                               const AttnArgs& args, int num_sms, cudaStream_t st) {
  return args.mode == 1 ? launch_attention_freq<T>(mq, mk, mv, args, num_sms, st)
                        : launch_attention_time<T>(mq, mk, mv, args, num_sms, st);
}

}  // namespace

cudaError_t launch_gemm(int epi, int precision, const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap* mo,
                        const GemmArgs& args, int num_sms, cudaStream_t st) {
  return precision == 0 ? launch_gemm_p<__half>(epi, ma, mb, mo, args, num_sms, st)
                        : launch_gemm_p<__nv_bfloat16>(epi, ma, mb, mo, args, num_sms, st);
}

template <typename T>
cudaError_t launch_mlp_t(const CUtensorMap& ma, const CUtensorMap& mw1, const CUtensorMap& mw2, const CUtensorMap& mx,
                         const CUtensorMap& mxn, const MlpArgs& args, int num_sms, cudaStream_t st) {
  auto kern = mlp_kernel<T>;
  static std::atomic<unsigned long long> done{0};  // one per <T> instantiation
  cudaError_t e = allow_smem(kern, MlpSmem::kBytes, done);
  if (e != cudaSuccess) return e;
  if (args.num_blocks <= 0) return cudaSuccess;
  const int grid = args.num_blocks < num_sms ? args.num_blocks : num_sms;
  kern<<<grid, kMlpThreads, MlpSmem::kBytes, st>>>(ma, mw1, mw2, mx, mxn, args);
  return cudaGetLastError();
}

cudaError_t launch_mlp(int precision, const CUtensorMap& ma, const CUtensorMap& mw1, const CUtensorMap& mw2,
                       const CUtensorMap& mx, const CUtensorMap& mxn, const MlpArgs& args, int num_sms,
                       cudaStream_t st) {
  return precision == 0 ? launch_mlp_t<__half>(ma, mw1, mw2, mx, mxn, args, num_sms, st)
                        : launch_mlp_t<__nv_bfloat16>(ma, mw1, mw2, mx, mxn, args, num_sms, st);
}

cudaError_t launch_attention(int precision, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const AttnArgs& args, int num_sms, cudaStream_t st) {
  return precision == 0 ? launch_attention_t<__half>(mq, mk, mv, args, num_sms, st)
                        : launch_attention_t<__nv_bfloat16>(mq, mk, mv, args, num_sms, st);
}

}  // namespace trc
