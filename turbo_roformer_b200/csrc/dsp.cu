// fp32 signal-processing kernels around the transformer: STFT, band split, row L2-norm, mask apply +
// iSTFT, and the Hamming overlap-add of chunk outputs. All HBM-bound; each thread block owns whole
// frames / rows so every global access is coalesced and every intermediate stays in shared memory.
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"
#include "sm100.cuh"

namespace trc {

// ------------------------------------------------------------------------------------------------ FFT
// In-place iterative radix-2 FFT of N = 2^log2n complex values in shared memory that were stored in
// bit-reversed order. tw[k] = exp(sign * 2 pi i k / N), k < N/2 (computed on the host in fp64).
__device__ __forceinline__ void fft_smem(float2* buf, const float2* __restrict__ tw, int n, int log2n) {
  for (int s = 1; s <= log2n; ++s) {
    const int half = 1 << (s - 1);
    const int tstride = n >> s;
    for (int j = threadIdx.x; j < (n >> 1); j += blockDim.x) {
      const int pos = j & (half - 1);
      const int i0 = ((j >> (s - 1)) << s) + pos;
      const int i1 = i0 + half;
      const float2 w = __ldg(&tw[pos * tstride]);
      const float2 a = buf[i0];
      const float2 b = buf[i1];
      const float2 bw = make_float2(b.x * w.x - b.y * w.y, b.x * w.y + b.y * w.x);
      buf[i0] = make_float2(a.x + bw.x, a.y + bw.y);
      buf[i1] = make_float2(a.x - bw.x, a.y - bw.y);
    }
    __syncthreads();
  }
}

__device__ __forceinline__ int bitrev(int k, int log2n) { return (int)(__brev((unsigned)k) >> (32 - log2n)); }

// STFT of one frame of both channels (torch.stft: center=True reflect padding, periodic Hann window,
// onesided, unnormalised; turbo_roformer/model.py:231-234, fast.py:370-376). The two real channels
// are packed as x0 + i x1 into one complex FFT and separated afterwards.
// audio [B][2][L]; xin [B*T][nf][2 ch][re, im] with nf = N/2 + 1.
__global__ void stft_kernel(const float* __restrict__ audio, int64_t L, int T, int n, int log2n, int hop,
                            const float* __restrict__ window, const float2* __restrict__ tw, float* __restrict__ xin) {
  extern __shared__ float2 fbuf[];
  const int bt = blockIdx.x;
  const int b = bt / T, t = bt - b * T;
  const float* x0 = audio + (size_t)b * 2 * L;
  const float* x1 = x0 + L;
  for (int k = threadIdx.x; k < n; k += blockDim.x) {
    int64_t i = (int64_t)t * hop + k - (n >> 1);
    if (i < 0) i = -i;
    if (i >= L) i = 2 * (L - 1) - i;
    const float w = window[k];
    fbuf[bitrev(k, log2n)] = make_float2(x0[i] * w, x1[i] * w);
  }
  __syncthreads();
  fft_smem(fbuf, tw, n, log2n);
  const int nf = (n >> 1) + 1;
  float4* out = reinterpret_cast<float4*>(xin + (size_t)bt * nf * 4);
  for (int f = threadIdx.x; f < nf; f += blockDim.x) {
    const float2 z = fbuf[f];
    const float2 zc = fbuf[(n - f) & (n - 1)];
    // X0 = (Z + conj Zr) / 2 ; X1 = (Z - conj Zr) / 2i
    const float x0r = 0.5f * (z.x + zc.x), x0i = 0.5f * (z.y - zc.y);
    const float x1r = 0.5f * (z.y + zc.y), x1i = -0.5f * (z.x - zc.x);
    out[f] = make_float4(x0r, x0i, x1r, x1i);
  }
}

// Mask apply + inverse real FFT + synthesis window for one frame of both channels
// (turbo_roformer/fast.py:388-393; torch.istft with irfft "backward" scaling). Bins 0 and N/2 use their
// real part only, as a complex-to-real transform does. frames [B*T][2][N] (windowed, not yet summed).
__global__ void istft_frames_kernel(const float* __restrict__ xin, const float* __restrict__ mask, int n, int log2n,
                                    const float* __restrict__ window, const float2* __restrict__ tw_inv,
                                    float* __restrict__ frames) {
  extern __shared__ float2 fbuf[];
  const int bt = blockIdx.x;
  const int nf = (n >> 1) + 1;
  const float4* sp = reinterpret_cast<const float4*>(xin + (size_t)bt * nf * 4);
  const float4* mp = reinterpret_cast<const float4*>(mask + (size_t)bt * nf * 4);
  for (int f = threadIdx.x; f < nf; f += blockDim.x) {
    const float4 s = sp[f], m = mp[f];
    float y0r = s.x * m.x - s.y * m.y, y0i = s.x * m.y + s.y * m.x;
    float y1r = s.z * m.z - s.w * m.w, y1i = s.z * m.w + s.w * m.z;
    if (f == 0 || f == nf - 1) {
      y0i = 0.f;
      y1i = 0.f;
    }
    // Z = Y0 + i Y1 over the Hermitian-extended spectra
    fbuf[bitrev(f, log2n)] = make_float2(y0r - y1i, y0i + y1r);
    if (f != 0 && f != nf - 1) fbuf[bitrev(n - f, log2n)] = make_float2(y0r + y1i, y1r - y0i);
  }
  __syncthreads();
  fft_smem(fbuf, tw_inv, n, log2n);
  const float inv_n = 1.0f / (float)n;
  float* o0 = frames + (size_t)bt * 2 * n;
  float* o1 = o0 + n;
  for (int k = threadIdx.x; k < n; k += blockDim.x) {
    const float2 z = fbuf[k];
    const float w = window[k];
    o0[k] = z.x * inv_n * w;
    o1[k] = z.y * inv_n * w;
  }
}

// Overlap-add of the windowed frames and division by the summed squared window, trimmed by N/2 on
// both sides (torch.istft center=True). out [B][2][hop * (T - 1)].
__global__ void istft_ola_kernel(const float* __restrict__ frames, int B, int T, int n, int hop,
                                 const float* __restrict__ window, float* __restrict__ out, int64_t lout) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)B * lout) return;
  const int b = (int)(idx / lout);
  const int64_t i = idx - (int64_t)b * lout;
  const int64_t p = i + (n >> 1);
  int64_t t_hi = p / hop;
  if (t_hi > T - 1) t_hi = T - 1;
  int64_t t_lo = p - n + 1 <= 0 ? 0 : (p - n + 1 + hop - 1) / hop;
  float s0 = 0.f, s1 = 0.f, env = 0.f;
  for (int64_t t = t_lo; t <= t_hi; ++t) {
    const int k = (int)(p - t * hop);
    const float* fr = frames + ((size_t)b * T + t) * 2 * n;
    const float w = window[k];
    s0 += fr[k];
    s1 += fr[n + k];
    env += w * w;
  }
  out[(size_t)b * 2 * lout + i] = s0 / env;
  out[(size_t)b * 2 * lout + lout + i] = s1 / env;
}

// Band split (turbo_roformer/model.py:147-155): per band k, X = W'_k x / max(|x|, 1e-12) + b_k with the
// RMSNorm gain sqrt(din) * gamma folded into W'. One block = 64 rows (batch x frame) of one band;
// thread o = output feature. wt [sum din][256] (transposed, folded), bias [nbands][256],
// X [rows][nbands][256] fp32.
// R rows (frames) x one band x 256 outputs per block: a thread owns one output column for R rows; small R
// gives many short blocks, which balances the very different band widths (8 to 512 inputs) over the SMs.
template <int R>
__global__ void __launch_bounds__(256) band_split_kernel(const float* __restrict__ xin, int width, int rows,
                                                         int nbands, const int* __restrict__ band_off,
                                                         const float* __restrict__ wt, const float* __restrict__ bias,
                                                         float* __restrict__ X) {
  __shared__ __align__(16) float xs[R][68];  // row stride 68 keeps float4 reads 16-byte aligned
  __shared__ float ssq_s[R];
  const int band = blockIdx.y;
  const int r0 = blockIdx.x * R;
  const int off = band_off[band];
  const int din = band_off[band + 1] - off;  // 4 * bins: always a multiple of 4
  const int o = threadIdx.x;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  float ssq = 0.f;
  for (int c0 = 0; c0 < din; c0 += 64) {
    const int cw = min(64, din - c0);
#pragma unroll 4
    for (int k = 0; k < R / 4; ++k) {
      const int e = o + k * 256;
      const int row = e >> 6, col = e & 63;
      float v = 0.f;
      if (r0 + row < rows && col < cw) v = xin[(size_t)(r0 + row) * width + off + c0 + col];
      xs[row][col] = v;
    }
    __syncthreads();
    if (o < R) {
      for (int col = 0; col < cw; ++col) ssq += xs[o][col] * xs[o][col];
    }
    for (int i = 0; i < cw; i += 4) {
      const float* wp = wt + (size_t)(off + c0 + i) * 256 + o;
      const float w0 = wp[0], w1 = wp[256], w2 = wp[512], w3 = wp[768];
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float4 xv = *reinterpret_cast<const float4*>(&xs[r][i]);
        acc[r] = fmaf(xv.w, w3, fmaf(xv.z, w2, fmaf(xv.y, w1, fmaf(xv.x, w0, acc[r]))));
      }
    }
    __syncthreads();
  }
  if (o < R) ssq_s[o] = ssq;
  __syncthreads();
  const float bo = bias[band * 256 + o];
#pragma unroll 4
  for (int r = 0; r < R; ++r) {
    const int row = r0 + r;
    if (row < rows) {
      const float inv = 1.0f / fmaxf(sqrtf(ssq_s[r]), 1e-12f);
      X[((size_t)row * nbands + band) * 256 + o] = acc[r] * inv + bo;
    }
  }
}

// xn = X / max(|X|, eps) per 256-feature row (turbo_roformer/csrc/kernels.cpp:102-137, without the add).
// One warp per row.
template <typename TOut>
__global__ void rownorm_kernel(const float* __restrict__ X, TOut* __restrict__ xn, int64_t rows, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(X + row * 256);
  const float4 a = xr[lane], b = xr[32 + lane];
  float ss = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  const float inv = 1.0f / fmaxf(sqrtf(ss), eps);
  TOut* o = xn + row * 256;
  uint2* o2 = reinterpret_cast<uint2*>(o);
  o2[lane] = make_uint2(OperandType<TOut>::pack2(a.x * inv, a.y * inv), OperandType<TOut>::pack2(a.z * inv, a.w * inv));
  o2[32 + lane] =
      make_uint2(OperandType<TOut>::pack2(b.x * inv, b.y * inv), OperandType<TOut>::pack2(b.z * inv, b.w * inv));
}

// X (+)= Y ; out = X / max(|X|, eps) as fp32 (out_f32) or 16-bit. One warp per row.
template <typename TOut>
__global__ void add_rmsnorm_kernel(float* __restrict__ X, const float* __restrict__ Y, void* __restrict__ out,
                                   int out_f32, int64_t rows, float eps) {
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float4* xr = reinterpret_cast<float4*>(X + row * 256);
  float4 a = xr[lane], b = xr[32 + lane];
  if (Y) {
    const float4* yr = reinterpret_cast<const float4*>(Y + row * 256);
    const float4 ya = yr[lane], yb = yr[32 + lane];
    a.x += ya.x; a.y += ya.y; a.z += ya.z; a.w += ya.w;
    b.x += yb.x; b.y += yb.y; b.z += yb.z; b.w += yb.w;
    xr[lane] = a;
    xr[32 + lane] = b;
  }
  float ss = a.x * a.x + a.y * a.y + a.z * a.z + a.w * a.w + b.x * b.x + b.y * b.y + b.z * b.z + b.w * b.w;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  const float inv = 1.0f / fmaxf(sqrtf(ss), eps);
  if (out_f32) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + row * 256);
    o[lane] = make_float4(a.x * inv, a.y * inv, a.z * inv, a.w * inv);
    o[32 + lane] = make_float4(b.x * inv, b.y * inv, b.z * inv, b.w * inv);
  } else {
    uint2* o2 = reinterpret_cast<uint2*>(static_cast<TOut*>(out) + row * 256);
    o2[lane] =
        make_uint2(OperandType<TOut>::pack2(a.x * inv, a.y * inv), OperandType<TOut>::pack2(a.z * inv, a.w * inv));
    o2[32 + lane] =
        make_uint2(OperandType<TOut>::pack2(b.x * inv, b.y * inv), OperandType<TOut>::pack2(b.z * inv, b.w * inv));
  }
}

// Hamming-weighted overlap-add of chunk outputs (turbo_roformer/chunking.py:54-61). For each sample the
// covering chunks form a contiguous range of the (increasing) starts; they are summed in start order
// with separately rounded multiply and add, so the result equals the reference's sequential
// `result += y * w; weight += w; result / max(weight, 1e-10)` bit for bit.
// chunks [n_chunks][2][clen]; out [2][n].
__global__ void chunk_ola_kernel(const float* __restrict__ chunks, int64_t clen, const int64_t* __restrict__ starts,
                                 int n_chunks, const float* __restrict__ w, int64_t n, float* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  // hi = last chunk with start <= i ; lo = first chunk with start > i - clen
  int lo = 0, hi = n_chunks - 1;
  {
    int a = 0, b = n_chunks - 1, res = -1;
    while (a <= b) {
      const int mid = (a + b) >> 1;
      if (starts[mid] <= i) { res = mid; a = mid + 1; } else { b = mid - 1; }
    }
    hi = res;
  }
  {
    int a = 0, b = n_chunks - 1, res = n_chunks;
    while (a <= b) {
      const int mid = (a + b) >> 1;
      if (starts[mid] > i - clen) { res = mid; b = mid - 1; } else { a = mid + 1; }
    }
    lo = res;
  }
  float r0 = 0.f, r1 = 0.f, ws = 0.f;
  for (int c = lo; c <= hi; ++c) {
    const int64_t k = i - starts[c];
    const float wv = w[k];
    const float* y = chunks + (size_t)c * 2 * clen;
    r0 = __fadd_rn(r0, __fmul_rn(y[k], wv));
    r1 = __fadd_rn(r1, __fmul_rn(y[clen + k], wv));
    ws = __fadd_rn(ws, wv);
  }
  const float d = fmaxf(ws, 1e-10f);
  out[i] = __fdiv_rn(r0, d);
  out[n + i] = __fdiv_rn(r1, d);
}

// ------------------------------------------------------------------------------------------------ launchers
void launch_stft(const float* audio, int B, int64_t L, int T, int n, int hop, const float* window, const float2* tw,
                 float* xin, cudaStream_t st) {
  const int log2n = __builtin_ctz(n);
  stft_kernel<<<B * T, 256, n * sizeof(float2), st>>>(audio, L, T, n, log2n, hop, window, tw, xin);
}

void launch_istft(const float* xin, const float* mask, int B, int T, int n, int hop, const float* window,
                  const float2* tw_inv, float* frames, float* out, cudaStream_t st) {
  const int log2n = __builtin_ctz(n);
  istft_frames_kernel<<<B * T, 256, n * sizeof(float2), st>>>(xin, mask, n, log2n, window, tw_inv, frames);
  const int64_t lout = (int64_t)hop * (T - 1);
  const int64_t total = (int64_t)B * lout;
  istft_ola_kernel<<<(unsigned)((total + 255) / 256), 256, 0, st>>>(frames, B, T, n, hop, window, out, lout);
}

void launch_band_split(const float* xin, int width, int rows, int nbands, const int* band_off, const float* wt,
                       const float* bias, float* X, cudaStream_t st) {
  dim3 grid((rows + 15) / 16, nbands);
  band_split_kernel<16><<<grid, 256, 0, st>>>(xin, width, rows, nbands, band_off, wt, bias, X);
}

void launch_rownorm(const float* X, void* xn, int64_t rows, float eps, int precision, cudaStream_t st) {
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (precision == 0)
    rownorm_kernel<__half><<<blocks, 256, 0, st>>>(X, static_cast<__half*>(xn), rows, eps);
  else
    rownorm_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(X, static_cast<__nv_bfloat16*>(xn), rows, eps);
}

void launch_add_rmsnorm(float* X, const float* Y, void* out, int out_f32, int64_t rows, float eps, int precision,
                        cudaStream_t st) {
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (precision == 0)
    add_rmsnorm_kernel<__half><<<blocks, 256, 0, st>>>(X, Y, out, out_f32, rows, eps);
  else
    add_rmsnorm_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(X, Y, out, out_f32, rows, eps);
}

// Self-test of the bounded-wait error path every pipelined kernel relies on: one thread waits on a
// shared-memory barrier that nothing will signal; after the wait limit it records kErrWaitSelftest in
// the error word and returns, leaving the context usable. No fault, no trap, no hang.
__global__ void wait_timeout_selftest_kernel(int* err) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) mbar_wait(&bar, 0, err, kErrWaitSelftest, &abort_flag);
}

void launch_wait_timeout_selftest(int* err, cudaStream_t st) { wait_timeout_selftest_kernel<<<1, 32, 0, st>>>(err); }

void launch_chunk_ola(const float* chunks, int64_t clen, const int64_t* d_starts, int n_chunks, const float* w,
                      int64_t n, float* out, cudaStream_t st) {
  chunk_ola_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(chunks, clen, d_starts, n_chunks, w, n, out);
}

}  // namespace trc
