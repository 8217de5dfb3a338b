// fp32 signal-processing kernels around the transformer: STFT, band split, row L2-norm, mask apply +
// iSTFT, and the Hamming overlap-add of chunk outputs. All HBM-bound; each thread block owns whole
// frames / rows so every global access is coalesced and every intermediate stays in shared memory.
#include <algorithm>
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
// Two consecutive radix-2 stages (s and s + 1) are done as one radix-4 pass: each thread takes the four
// values a stage-s butterfly pair and its partner pair feed into, so every value is read and written
// once per two stages and the block synchronises half as often. The arithmetic per output is the
// radix-2 stages' own.
__device__ __forceinline__ float2 cmul(float2 b, float2 w) {
  return make_float2(b.x * w.x - b.y * w.y, b.x * w.y + b.y * w.x);
}

__device__ __forceinline__ void fft_smem(float2* buf, const float2* __restrict__ tw, int n, int log2n) {
  int s = 1;
  for (; s + 1 <= log2n; s += 2) {
    const int h = 1 << (s - 1);  // stage-s butterfly distance; stage s + 1 uses 2h
    for (int j = threadIdx.x; j < (n >> 2); j += blockDim.x) {
      const int pos = j & (h - 1);
      const int i0 = ((j >> (s - 1)) << (s + 1)) + pos;
      const float2 w1 = __ldg(&tw[pos * (n >> s)]);             // W_{2h}^pos
      const float2 w2 = __ldg(&tw[pos * (n >> (s + 1))]);       // W_{4h}^pos
      const float2 w3 = __ldg(&tw[(pos + h) * (n >> (s + 1))]);  // W_{4h}^(pos + h)
      const float2 a = buf[i0], b = buf[i0 + h], c = buf[i0 + 2 * h], d = buf[i0 + 3 * h];
      const float2 bw = cmul(b, w1), dw = cmul(d, w1);
      const float2 a1 = make_float2(a.x + bw.x, a.y + bw.y), b1 = make_float2(a.x - bw.x, a.y - bw.y);
      const float2 c1 = make_float2(c.x + dw.x, c.y + dw.y), d1 = make_float2(c.x - dw.x, c.y - dw.y);
      const float2 cw = cmul(c1, w2), dw2 = cmul(d1, w3);
      buf[i0] = make_float2(a1.x + cw.x, a1.y + cw.y);
      buf[i0 + 2 * h] = make_float2(a1.x - cw.x, a1.y - cw.y);
      buf[i0 + h] = make_float2(b1.x + dw2.x, b1.y + dw2.y);
      buf[i0 + 3 * h] = make_float2(b1.x - dw2.x, b1.y - dw2.y);
    }
    __syncthreads();
  }
  if (s == log2n) {  // odd number of stages: a last radix-2 stage
    const int half = 1 << (s - 1);
    for (int j = threadIdx.x; j < (n >> 1); j += blockDim.x) {
      const int pos = j & (half - 1);
      const int i0 = ((j >> (s - 1)) << s) + pos;
      const int i1 = i0 + half;
      const float2 w = __ldg(&tw[pos * (n >> s)]);
      const float2 a = buf[i0];
      const float2 bw = cmul(buf[i1], w);
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

// Band-split inputs of one frame for the grouped band-split GEMM (turbo_roformer/model.py:147-155): each
// band's 4 * bins values divided by their L2 norm (F.normalize inside the band's RMSNorm, eps 1e-12; the
// sqrt(din) * gamma gain is folded into the GEMM's weights), rounded to the operand type, each band
// starting at a multiple of 64 columns and zero-padded up to the next one.
// xin [rows][width] fp32 (band k at columns band_off[k] ..); a [rows][kp] 16-bit (band k at pad_off[k]).
// One block per frame; its warps take the bands in turn.
template <typename TOut>
__global__ void __launch_bounds__(256) band_pack_kernel(const float* __restrict__ xin, int width, int nbands,
                                                        const int* __restrict__ band_off,
                                                        const int* __restrict__ pad_off, int kp,
                                                        TOut* __restrict__ a) {
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float* x = xin + (size_t)row * width;
  TOut* o = a + (size_t)row * kp;
  for (int k = warp; k < nbands; k += blockDim.x >> 5) {
    const int off = band_off[k], din = band_off[k + 1] - off;
    const int po = pad_off[k], pw = pad_off[k + 1] - po;
    float ss = 0.f;
    for (int c = lane; c < din; c += 32) {
      const float v = x[off + c];
      ss = fmaf(v, v, ss);
    }
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
    const float inv = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
    for (int c = lane; c < pw; c += 32) o[po + c] = OperandType<TOut>::from_float(c < din ? x[off + c] * inv : 0.f);
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

// Rows of any width 64 * M (models whose width is not 256): X (+)= Y, out = X / max(|X|, eps), one warp
// per row, lane l holding the float2s l, l + 32, ... of the row (every access a coalesced 256-byte row
// segment per warp).
template <typename TOut, int M>
__global__ void add_rmsnorm_d_kernel(float* __restrict__ X, const float* __restrict__ Y, void* __restrict__ out,
                                     int out_f32, int64_t rows, float eps) {
  constexpr int D = 64 * M;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  float2* xr = reinterpret_cast<float2*>(X + row * D);
  float2 v[M];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < M; ++i) {
    v[i] = xr[i * 32 + lane];
    if (Y) {
      const float2 y = reinterpret_cast<const float2*>(Y + row * D)[i * 32 + lane];
      v[i].x += y.x;
      v[i].y += y.y;
      xr[i * 32 + lane] = v[i];
    }
    ss += v[i].x * v[i].x + v[i].y * v[i].y;
  }
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, d);
  const float inv = 1.0f / fmaxf(sqrtf(ss), eps);
#pragma unroll
  for (int i = 0; i < M; ++i) {
    if (out_f32)
      reinterpret_cast<float2*>(static_cast<float*>(out) + row * D)[i * 32 + lane] = make_float2(v[i].x * inv, v[i].y * inv);
    else
      reinterpret_cast<uint32_t*>(static_cast<TOut*>(out) + row * D)[i * 32 + lane] =
          OperandType<TOut>::pack2(v[i].x * inv, v[i].y * inv);
  }
}

template <typename TOut, int M>
void launch_norm_m(float* X, const float* Y, void* out, int out_f32, int64_t rows, float eps, cudaStream_t st) {
  add_rmsnorm_d_kernel<TOut, M><<<(unsigned)((rows + 7) / 8), 256, 0, st>>>(X, Y, out, out_f32, rows, eps);
}

template <typename TOut>
void launch_add_rmsnorm_d(float* X, const float* Y, void* out, int out_f32, int64_t rows, float eps, int dim,
                          cudaStream_t st) {
  switch (dim / 64) {  // dim is a multiple of 64 in [128, 1024] (checked by trc_create)
    case 2: launch_norm_m<TOut, 2>(X, Y, out, out_f32, rows, eps, st); break;
    case 3: launch_norm_m<TOut, 3>(X, Y, out, out_f32, rows, eps, st); break;
    case 4: launch_norm_m<TOut, 4>(X, Y, out, out_f32, rows, eps, st); break;
    case 5: launch_norm_m<TOut, 5>(X, Y, out, out_f32, rows, eps, st); break;
    case 6: launch_norm_m<TOut, 6>(X, Y, out, out_f32, rows, eps, st); break;
    case 7: launch_norm_m<TOut, 7>(X, Y, out, out_f32, rows, eps, st); break;
    case 8: launch_norm_m<TOut, 8>(X, Y, out, out_f32, rows, eps, st); break;
    case 9: launch_norm_m<TOut, 9>(X, Y, out, out_f32, rows, eps, st); break;
    case 10: launch_norm_m<TOut, 10>(X, Y, out, out_f32, rows, eps, st); break;
    case 11: launch_norm_m<TOut, 11>(X, Y, out, out_f32, rows, eps, st); break;
    case 12: launch_norm_m<TOut, 12>(X, Y, out, out_f32, rows, eps, st); break;
    case 13: launch_norm_m<TOut, 13>(X, Y, out, out_f32, rows, eps, st); break;
    case 14: launch_norm_m<TOut, 14>(X, Y, out, out_f32, rows, eps, st); break;
    case 15: launch_norm_m<TOut, 15>(X, Y, out, out_f32, rows, eps, st); break;
    default: launch_norm_m<TOut, 16>(X, Y, out, out_f32, rows, eps, st); break;
  }
}

// Hamming-weighted overlap-add of chunk outputs (turbo_roformer/chunking.py:54-61). For each sample the
// covering chunks form a contiguous range of the (increasing) starts; they are summed in start order
// with separately rounded multiply and add, so the result equals the reference's sequential
// `result += y * w; weight += w; result / max(weight, 1e-10)` bit for bit.
// chunks [n_chunks][2][clen]; out [2][n].
// A block owns kOlaPerThread consecutive samples per thread, laid out block-strided (sample
// i0 + s * blockDim.x + threadIdx.x for s < kOlaPerThread) so every load and store stays coalesced; one
// pair of binary searches per block finds the chunks that cover the block's span, and each sample then
// walks that short range, skipping chunks that do not cover it.
constexpr int kOlaPerThread = 8;

__global__ void __launch_bounds__(256) chunk_ola_kernel(const float* __restrict__ chunks, int64_t clen,
                                                        const int64_t* __restrict__ starts, int n_chunks,
                                                        const float* __restrict__ w, int64_t n,
                                                        float* __restrict__ out) {
  __shared__ int range[2];
  const int64_t i0 = (int64_t)blockIdx.x * blockDim.x * kOlaPerThread;
  const int64_t i1 = min(n, i0 + (int64_t)blockDim.x * kOlaPerThread) - 1;  // last sample of the block
  if (threadIdx.x == 0) {
    // hi = last chunk with start <= i1 ; lo = first chunk with start > i0 - clen
    int a = 0, b = n_chunks - 1, res = -1;
    while (a <= b) {
      const int mid = (a + b) >> 1;
      if (starts[mid] <= i1) { res = mid; a = mid + 1; } else { b = mid - 1; }
    }
    range[1] = res;
    a = 0, b = n_chunks - 1, res = n_chunks;
    while (a <= b) {
      const int mid = (a + b) >> 1;
      if (starts[mid] > i0 - clen) { res = mid; b = mid - 1; } else { a = mid + 1; }
    }
    range[0] = res;
  }
  __syncthreads();
  const int lo = range[0], hi = range[1];
#pragma unroll
  for (int s = 0; s < kOlaPerThread; ++s) {
    const int64_t i = i0 + (int64_t)s * blockDim.x + threadIdx.x;
    if (i >= n) break;
    float r0 = 0.f, r1 = 0.f, ws = 0.f;
    for (int c = lo; c <= hi; ++c) {
      const int64_t k = i - starts[c];
      if (k < 0 || k >= clen) continue;  // chunk c does not cover sample i
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

void launch_band_pack(const float* xin, int width, int rows, int nbands, const int* band_off, const int* pad_off,
                      int kp, void* a, int precision, cudaStream_t st) {
  if (precision == 0)
    band_pack_kernel<__half><<<rows, 256, 0, st>>>(xin, width, nbands, band_off, pad_off, kp, static_cast<__half*>(a));
  else
    band_pack_kernel<__nv_bfloat16>
        <<<rows, 256, 0, st>>>(xin, width, nbands, band_off, pad_off, kp, static_cast<__nv_bfloat16*>(a));
}

void launch_rownorm(const float* X, void* xn, int64_t rows, float eps, int precision, int dim, cudaStream_t st) {
  if (dim != 256) {
    if (precision == 0)
      launch_add_rmsnorm_d<__half>(const_cast<float*>(X), nullptr, xn, 0, rows, eps, dim, st);
    else
      launch_add_rmsnorm_d<__nv_bfloat16>(const_cast<float*>(X), nullptr, xn, 0, rows, eps, dim, st);
    return;
  }
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (precision == 0)
    rownorm_kernel<__half><<<blocks, 256, 0, st>>>(X, static_cast<__half*>(xn), rows, eps);
  else
    rownorm_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(X, static_cast<__nv_bfloat16*>(xn), rows, eps);
}

void launch_add_rmsnorm(float* X, const float* Y, void* out, int out_f32, int64_t rows, float eps, int precision,
                        int dim, cudaStream_t st) {
  if (dim != 256) {
    if (precision == 0)
      launch_add_rmsnorm_d<__half>(X, Y, out, out_f32, rows, eps, dim, st);
    else
      launch_add_rmsnorm_d<__nv_bfloat16>(X, Y, out, out_f32, rows, eps, dim, st);
    return;
  }
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
  const int64_t per_block = 256 * kOlaPerThread;
  chunk_ola_kernel<<<(unsigned)((n + per_block - 1) / per_block), 256, 0, st>>>(chunks, clen, d_starts, n_chunks, w,
                                                                                 n, out);
}

// ------------------------------------------------------------------------------------------ remix / resample
// Channel fold to stereo (audio.downmix_stereo / to_stereo, turbo_roformer/audio.py:35-68): one output
// sample per thread and side, the channel sum in fp64 in channel order with separately rounded products
// and sums (the host fold's operations, so both agree bit for bit), rounded once to fp32.
struct RemixGains {
  double g[2][kRemixMaxChannels];
};

__global__ void __launch_bounds__(256) remix_kernel(const float* __restrict__ x, int channels, int64_t n,
                                                    const RemixGains gains, float* __restrict__ y) {
  const int side = blockIdx.y;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    double acc = 0.0;
    for (int k = 0; k < channels; ++k) acc = __dadd_rn(acc, __dmul_rn(gains.g[side][k], (double)__ldg(x + (size_t)k * n + i)));
    y[(size_t)side * n + i] = (float)acc;
  }
}

// Rational-ratio polyphase FIR resampling (the role of audio.resample, turbo_roformer/audio.py:71-82):
// output m sits at t = m * down + half on the up-sampled grid; its taps are column p = t % up of the
// [K][up] table and its inputs x[j0 - k], j0 = t / up, k = 0..K-1 (zero outside [0, n_in)). One output
// per thread: a warp's outputs read neighbouring inputs (coalesced) and scattered columns of one tap row
// (L1/L2 resident). fp64 accumulation in k order, rounded once.
__global__ void __launch_bounds__(256) resample_kernel(const float* __restrict__ x, int64_t n_in, int up, int down,
                                                       int64_t half, const double* __restrict__ taps, int K,
                                                       int64_t n_out, float* __restrict__ y) {
  const float* xc = x + (size_t)blockIdx.y * n_in;
  float* yc = y + (size_t)blockIdx.y * n_out;
  for (int64_t m = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; m < n_out;
       m += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = m * down + half;
    const int64_t j0 = t / up;
    const int p = (int)(t - j0 * up);
    const int k0 = j0 >= n_in ? (int)min(j0 - n_in + 1, (int64_t)K) : 0;  // skip inputs past the end
    const int k1 = (int)min((int64_t)K, j0 + 1);                           // and before the start
    double acc = 0.0;
    for (int k = k0; k < k1; ++k) acc = fma(__ldg(taps + (size_t)k * up + p), (double)__ldg(xc + (j0 - k)), acc);
    yc[m] = (float)acc;
  }
}

void launch_remix(const float* x, int channels, int64_t n, const double* gains, float* y, cudaStream_t st) {
  RemixGains g;
  for (int side = 0; side < 2; ++side)
    for (int k = 0; k < kRemixMaxChannels; ++k) g.g[side][k] = k < channels ? gains[side * channels + k] : 0.0;
  const unsigned blocks = (unsigned)std::min<int64_t>((n + 255) / 256, 148 * 16);
  remix_kernel<<<dim3(blocks, 2), 256, 0, st>>>(x, channels, n, g, y);
}

void launch_resample(const float* x, int channels, int64_t n_in, int up, int down, int64_t half, const double* taps,
                     int K, int64_t n_out, float* y, cudaStream_t st) {
  const unsigned blocks = (unsigned)std::min<int64_t>((n_out + 255) / 256, 148 * 16);
  resample_kernel<<<dim3(blocks, channels), 256, 0, st>>>(x, n_in, up, down, half, taps, K, n_out, y);
}

}  // namespace trc
