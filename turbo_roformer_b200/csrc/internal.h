// Host-side launch interface shared by the translation units of libtrcuda.so (not part of the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace trc {

struct GemmArgs;
struct AttnArgs;
struct MlpArgs;

// api.cu: adds kernels launched outside api.cu to the count trc_launch_count reports
void count_launches(int n);

// dsp.cu
void launch_stft(const float* audio, int B, int64_t L, int T, int n, int hop, const float* window, const float2* tw,
                 float* xin, cudaStream_t st);
void launch_istft(const float* xin, const float* mask, int B, int T, int n, int hop, const float* window,
                  const float2* tw_inv, float* frames, float* out, cudaStream_t st);
void launch_band_pack(const float* xin, int width, int rows, int nbands, const int* band_off, const int* pad_off,
                      int kp, void* a, int precision, cudaStream_t st);
// rows of `dim` floats (a multiple of 64 in [128, 1024])
void launch_rownorm(const float* X, void* xn, int64_t rows, float eps, int precision, int dim, cudaStream_t st);
void launch_add_rmsnorm(float* X, const float* Y, void* out, int out_f32, int64_t rows, float eps, int precision,
                        int dim, cudaStream_t st);
void launch_wait_timeout_selftest(int* err, cudaStream_t st);
void launch_chunk_ola(const float* chunks, int64_t clen, const int64_t* d_starts, int n_chunks, const float* w,
                      int64_t n, float* out, cudaStream_t st);
constexpr int kRemixMaxChannels = 16;
void launch_remix(const float* x, int channels, int64_t n, const double* gains, float* y, cudaStream_t st);
void launch_resample(const float* x, int channels, int64_t n_in, int up, int down, int64_t half, const double* taps,
                     int K, int64_t n_out, float* y, cudaStream_t st);

// pack.cu (unfused attention-layout helpers)
void launch_rope_pack(int precision, const void* qkvg, const float* cos_tab, const float* sin_tab, int mode, int T,
                      int F, int64_t N, void* Q, void* K, void* V, float* G, cudaStream_t st);
void launch_gate_merge(int precision, const void* A, const float* G, void* O, int mode, int T, int F, int64_t N,
                       cudaStream_t st);

// tc.cu (tensor-core kernels). epi: EpiKind; precision: 0 fp16, 1 bf16; map_out: 3 output tensor maps
// (unused ones may hold anything). Return cudaError_t of the launch.
cudaError_t launch_gemm(int epi, int precision, const CUtensorMap& map_a, const CUtensorMap& map_b,
                        const CUtensorMap* map_out, const GemmArgs& args, int num_sms, cudaStream_t st);
cudaError_t launch_mlp(int precision, const CUtensorMap& ma, const CUtensorMap& mw1, const CUtensorMap& mw2,
                       const CUtensorMap& mx, const CUtensorMap& mxn, const MlpArgs& args, int num_sms,
                       cudaStream_t st);
cudaError_t launch_attention(int precision, const CUtensorMap& mq, const CUtensorMap& mk, const CUtensorMap& mv,
                             const AttnArgs& args, int num_sms, cudaStream_t st);

}  // namespace trc
