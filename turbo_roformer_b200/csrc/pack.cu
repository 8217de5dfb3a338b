// Unfused attention-layout helpers of the reference's op library, for callers that run the qkv GEMM or
// the attention itself elsewhere (the forward path fuses both into the GEMM and attention kernels):
//   rope_pack  (LoggeL/turbo-roformer src/turbo_roformer/csrc/kernels.cpp:161-248, packed = false):
//              qkv+gate GEMM output [N][1544] -> rotary q, k and plain v in the attention layout
//              [seq][L][64] plus G = sigmoid(gate logits) [N][8];
//   gate_merge (kernels.cpp:391-408): per-head attention output [seq][L][64] -> O[token][h*64 + d]
//              scaled by the head's gate.
// Token order is (b*T + t)*F + f; a time-mode sequence is (b, f, h) over t, a freq-mode sequence is
// (b, t, h) over f. One warp per (token or row, head); lane j owns the rotary pair (2j, 2j + 1), so every
// warp reads and writes one contiguous 128-byte head row. Both kernels are HBM bound.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "internal.h"

namespace trc {
namespace {

template <typename T>
struct Pair;
template <>
struct Pair<__half> {
  using V = __half2;
  __device__ static float2 to_f2(V v) { return __half22float2(v); }
  __device__ static V from_f2(float2 f) { return __floats2half2_rn(f.x, f.y); }
  __device__ static float to_f(__half v) { return __half2float(v); }
};
template <>
struct Pair<__nv_bfloat16> {
  using V = __nv_bfloat162;
  __device__ static float2 to_f2(V v) { return __bfloat1622float2(v); }
  __device__ static V from_f2(float2 f) { return __floats2bfloat162_rn(f.x, f.y); }
  __device__ static float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
};

// Sequence row of a token for one head: returns the element offset of the head row in [seq][L][64].
__device__ __forceinline__ int64_t head_row(int64_t tok, int h, int mode, int T, int F) {
  const int64_t bt = tok / F;
  const int f = (int)(tok - bt * F);
  const int64_t b = bt / T;
  const int t = (int)(bt - b * T);
  if (mode == 0) return (((b * F + f) * 8 + h) * T + t) * 64;
  return ((bt * 8 + h) * F + f) * 64;
}

template <typename TIn>
__global__ void __launch_bounds__(256) rope_pack_kernel(const TIn* __restrict__ qkvg, const float* __restrict__ cs,
                                                        const float* __restrict__ sn, int mode, int T, int F,
                                                        int64_t N, TIn* __restrict__ Q, TIn* __restrict__ K,
                                                        TIn* __restrict__ V, float* __restrict__ G) {
  using P = Pair<TIn>;
  const int64_t tok = blockIdx.x;
  if (tok >= N) return;
  const int h = threadIdx.x >> 5, j = threadIdx.x & 31;
  const int64_t bt = tok / F;
  const int pos = mode == 0 ? (int)(bt % T) : (int)(tok - bt * F);
  const float c = cs[pos * 32 + j], s = sn[pos * 32 + j];
  const TIn* src = qkvg + tok * 1544;
  const int64_t dst = head_row(tok, h, mode, T, F) + 2 * j;
  using V2 = typename P::V;
  // q and k: (x0, x1) -> (x0 c - x1 s, x1 c + x0 s) in fp32, rounded once
  const float2 q = P::to_f2(*reinterpret_cast<const V2*>(src + h * 64 + 2 * j));
  *reinterpret_cast<V2*>(Q + dst) = P::from_f2(make_float2(q.x * c - q.y * s, q.y * c + q.x * s));
  const float2 k = P::to_f2(*reinterpret_cast<const V2*>(src + 512 + h * 64 + 2 * j));
  *reinterpret_cast<V2*>(K + dst) = P::from_f2(make_float2(k.x * c - k.y * s, k.y * c + k.x * s));
  *reinterpret_cast<V2*>(V + dst) = *reinterpret_cast<const V2*>(src + 1024 + h * 64 + 2 * j);
  if (j == 0) G[tok * 8 + h] = 1.0f / (1.0f + expf(-P::to_f(src[1536 + h])));
}

template <typename TIn>
__global__ void __launch_bounds__(256) gate_merge_kernel(const TIn* __restrict__ A, const float* __restrict__ G,
                                                         TIn* __restrict__ O, int mode, int T, int F, int64_t rows,
                                                         int L) {
  using P = Pair<TIn>;
  using V2 = typename P::V;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const int64_t seq = row / L;
  const int pos = (int)(row - seq * L);
  const int h = (int)(seq & 7);
  const int64_t grp = seq >> 3;
  int64_t tok;
  if (mode == 0) {  // grp = b*F + f, pos = t
    const int64_t b = grp / F;
    tok = (b * T + pos) * F + (grp - b * F);
  } else {  // grp = b*T + t, pos = f
    tok = grp * F + pos;
  }
  const float g = G[tok * 8 + h];
  const float2 a = P::to_f2(*reinterpret_cast<const V2*>(A + row * 64 + 2 * lane));
  *reinterpret_cast<V2*>(O + tok * 512 + h * 64 + 2 * lane) = P::from_f2(make_float2(a.x * g, a.y * g));
}

}  // namespace

void launch_rope_pack(int precision, const void* qkvg, const float* cos_tab, const float* sin_tab, int mode, int T,
                      int F, int64_t N, void* Q, void* K, void* V, float* G, cudaStream_t st) {
  if (N <= 0) return;
  if (precision == 0)
    rope_pack_kernel<__half><<<(unsigned)N, 256, 0, st>>>(static_cast<const __half*>(qkvg), cos_tab, sin_tab, mode,
                                                          T, F, N, static_cast<__half*>(Q), static_cast<__half*>(K),
                                                          static_cast<__half*>(V), G);
  else
    rope_pack_kernel<__nv_bfloat16><<<(unsigned)N, 256, 0, st>>>(
        static_cast<const __nv_bfloat16*>(qkvg), cos_tab, sin_tab, mode, T, F, N, static_cast<__nv_bfloat16*>(Q),
        static_cast<__nv_bfloat16*>(K), static_cast<__nv_bfloat16*>(V), G);
}

void launch_gate_merge(int precision, const void* A, const float* G, void* O, int mode, int T, int F, int64_t N,
                       cudaStream_t st) {
  const int L = mode == 0 ? T : F;
  const int64_t rows = N * 8;  // (sequence, position) rows: N tokens x 8 heads
  if (rows <= 0) return;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (precision == 0)
    gate_merge_kernel<__half><<<blocks, 256, 0, st>>>(static_cast<const __half*>(A), G, static_cast<__half*>(O), mode,
                                                       T, F, rows, L);
  else
    gate_merge_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(static_cast<const __nv_bfloat16*>(A), G,
                                                              static_cast<__nv_bfloat16*>(O), mode, T, F, rows, L);
}

}  // namespace trc
