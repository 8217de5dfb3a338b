// Persistent tcgen05 GEMM  D[128 x BN] = A[128 x K] * B[BN x K]^T  with fused epilogues.
//
// Roles (192 threads):  warp 0 = TMA producer, warp 1 = MMA issuer + TMEM owner, warps 2-5 = epilogue.
// A and B are K-major 16-bit tiles (128-byte swizzle) streamed through a STAGES-deep shared-memory ring;
// the accumulator lives in TMEM, double buffered (2 x BN columns) so the epilogue of tile i overlaps the
// MMAs of tile i+1. Each epilogue thread owns one output row (TMEM lane), which makes row-wise epilogues
// (residual add + L2 norm over the 256 features of a token) thread-local.
//
// Epilogues (the reference kernels they replace, LoggeL/turbo-roformer src/turbo_roformer/csrc/kernels.cpp):
//   EPI_QKV       qkv_rope_gemm (:442-540): rotary on q,k in fp32, scatter to the attention layout, sigmoid gates
//   EPI_RESNORM   gemm_res_norm (:543-586): X += acc (+ bias); xn = X / max(|X|, eps)
//   EPI_GELU      gemm_gelu (:610-642):     H = gelu_erf(acc + b)
//   EPI_MASK_TANH mask MLP layer 1 (fast.py:354):  tanh(acc + b1) per band
//   EPI_MASK_GLU  mask MLP layer 2 + GLU (fast.py:355-357): a * sigmoid(g), with (a, g) rows interleaved
#pragma once

#include "sm100.cuh"

namespace trc {

enum EpiKind : int { EPI_QKV = 0, EPI_RESNORM = 1, EPI_GELU = 2, EPI_MASK_TANH = 3, EPI_MASK_GLU = 4 };

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kGemmThreads = 192;
constexpr int kMaxGroups = 64;

struct GemmArgs {
  // ---- schedule
  int num_tiles;
  int k_blocks;   // K / 64
  int a_mode;     // 0: A map 2D (k, row); 1: 3D (k, group, row); 2: 3D (k, row, group)
  int M;          // valid rows (per group when grouped)
  int n_tiles;    // dense: N tiles per M tile
  int N;          // dense: valid columns
  int n_groups;   // 0 = dense
  int g_tile_start[kMaxGroups + 1];
  int g_ntiles[kMaxGroups];
  int g_brow[kMaxGroups];    // first B row of the group
  int g_ncols[kMaxGroups];   // valid columns of the group
  int g_outoff[kMaxGroups];  // output column offset of the group (mask GLU)
  // ---- epilogue
  void* out0;
  void* out1;
  void* out2;
  void* out3;
  const float* bias;   // indexed by B row (nullptr = none)
  const float* bias2;  // qkv: gate bias [8]
  const float* cos_tab;
  const float* sin_tab;
  int T, F, mode, ld_out;
  float eps;
  int* err;
};

struct TileCoord {
  int m0, n0, group, b_row, n_valid, n_mma;
};

template <int BN>
__device__ __forceinline__ TileCoord gemm_decode(const GemmArgs& a, int tile) {
  TileCoord c;
  if (a.n_groups == 0) {
    const int mt = tile / a.n_tiles, nt = tile - mt * a.n_tiles;
    c.group = 0;
    c.m0 = mt * kGemmBM;
    c.n0 = nt * BN;
    c.b_row = c.n0;
    c.n_valid = min(BN, a.N - c.n0);
  } else {
    int g = 0;
    while (g + 1 < a.n_groups && tile >= a.g_tile_start[g + 1]) ++g;
    const int local = tile - a.g_tile_start[g];
    const int mt = local / a.g_ntiles[g], nt = local - mt * a.g_ntiles[g];
    c.group = g;
    c.m0 = mt * kGemmBM;
    c.n0 = nt * BN;
    c.b_row = a.g_brow[g] + c.n0;
    c.n_valid = min(BN, a.g_ncols[g] - c.n0);
  }
  c.n_mma = (c.n_valid + 15) & ~15;
  return c;
}

template <typename TIn>
__device__ __forceinline__ void store32(TIn* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint4 u;
    u.x = OperandType<TIn>::pack2(v[8 * i + 0], v[8 * i + 1]);
    u.y = OperandType<TIn>::pack2(v[8 * i + 2], v[8 * i + 3]);
    u.z = OperandType<TIn>::pack2(v[8 * i + 4], v[8 * i + 5]);
    u.w = OperandType<TIn>::pack2(v[8 * i + 6], v[8 * i + 7]);
    d[i] = u;
  }
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f)); }

// ------------------------------------------------------------------------------------------------ epilogues
// taddr: TMEM address of (this thread's lane, column 0 of the accumulator buffer). row valid iff m < M.
template <int BN, typename TIn>
__device__ __forceinline__ void epi_qkv(const GemmArgs& a, const TileCoord& tc, uint32_t taddr, int m, bool valid) {
  const int TF = a.T * a.F;
  const int b = m / TF;
  const int r = m - b * TF;
  const int t = r / a.F;
  const int f = r - t * a.F;
  int pos, L, bh0;
  if (a.mode == 0) {
    pos = t; L = a.T; bh0 = (b * a.F + f) * 8;
  } else {
    pos = f; L = a.F; bh0 = (b * a.T + t) * 8;
  }
  if (tc.n0 >= 1536) {  // gate columns: sigmoid(x . Wg + bg) -> G[token][8]
    float v[16];
    tmem_ld16(taddr, v);
    if (valid) {
      float g[8];
#pragma unroll
      for (int h = 0; h < 8; ++h) g[h] = sigmoidf_(v[h] + a.bias2[h]);
      float4* G = reinterpret_cast<float4*>(static_cast<float*>(a.out3) + (size_t)m * 8);
      G[0] = make_float4(g[0], g[1], g[2], g[3]);
      G[1] = make_float4(g[4], g[5], g[6], g[7]);
    }
    return;
  }
  const int part = tc.n0 >> 9;          // 0 q, 1 k, 2 v
  const int h0 = (tc.n0 & 511) >> 6;    // first head of this tile
  TIn* base = static_cast<TIn*>(part == 0 ? a.out0 : part == 1 ? a.out1 : a.out2);
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    tmem_ld32(taddr + c * 32, v);
    const int h = h0 + (c >> 1);
    const int d0 = (c & 1) * 32;
    if (part < 2 && valid) {
      const float4* cp = reinterpret_cast<const float4*>(a.cos_tab + (size_t)pos * 32 + (d0 >> 1));
      const float4* sp = reinterpret_cast<const float4*>(a.sin_tab + (size_t)pos * 32 + (d0 >> 1));
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 cs = cp[q], sn = sp[q];
        const float cc[4] = {cs.x, cs.y, cs.z, cs.w};
        const float ss[4] = {sn.x, sn.y, sn.z, sn.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = q * 4 + e;
          const float x0 = v[2 * i], x1 = v[2 * i + 1];
          v[2 * i] = x0 * cc[e] - x1 * ss[e];
          v[2 * i + 1] = x1 * cc[e] + x0 * ss[e];
        }
      }
    }
    if (valid) store32<TIn>(base + ((size_t)(bh0 + h) * L + pos) * 64 + d0, v);
  }
}

// Residual add + row L2 norm, warp-cooperative: the warp's 32 rows x 256 columns are moved through a
// padded shared-memory transpose 32 columns at a time, so X and xn are read and written as coalesced
// 128-byte row segments (one row per instruction, all 32 rows' loads in flight before any store).
// Per-lane partial sums of squares (one per row) are combined with a 31-shuffle transpose-reduce that
// leaves the total of row `lane` in lane `lane`.
template <int BN, typename TIn>
__device__ __forceinline__ void epi_resnorm(const GemmArgs& a, uint32_t taddr, int row0, int lane,
                                            float* stage) {
  float* X = static_cast<float*>(a.out0);
  TIn* xn = static_cast<TIn*>(a.out1);
  const int nrows = min(32, a.M - row0);  // rows of this warp that exist (may be <= 0)
  float ps[32];
#pragma unroll
  for (int r = 0; r < 32; ++r) ps[r] = 0.f;
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    float v[32];
    tmem_ld32(taddr + c * 32, v);
#pragma unroll
    for (int i = 0; i < 32; ++i) stage[lane * 33 + i] = v[i];
    __syncwarp();
    const int col = c * 32 + lane;
    const float b = a.bias ? a.bias[col] : 0.f;
    float x[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) x[r] = r < nrows ? X[(size_t)(row0 + r) * 256 + col] : 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      x[r] += stage[r * 33 + lane] + b;
      ps[r] = fmaf(x[r], x[r], ps[r]);
    }
#pragma unroll
    for (int r = 0; r < 32; ++r)
      if (r < nrows) X[(size_t)(row0 + r) * 256 + col] = x[r];
    __syncwarp();
  }
  // transpose-reduce: after the step with offset o, ps[i] (i < o) holds the pair-sum of the row
  // selected by the lane bits above o
#pragma unroll
  for (int o = 16; o >= 1; o >>= 1) {
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < o; ++i) {
      const float send = upper ? ps[i] : ps[i + o];
      const float keep = upper ? ps[i + o] : ps[i];
      ps[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  const float inv = 1.0f / fmaxf(sqrtf(ps[0]), a.eps);  // for row `lane`
#pragma unroll 1
  for (int c = 0; c < 8; ++c) {
    const int col = c * 32 + lane;
    float x[32];
#pragma unroll
    for (int r = 0; r < 32; ++r) x[r] = r < nrows ? X[(size_t)(row0 + r) * 256 + col] : 0.f;
#pragma unroll
    for (int r = 0; r < 32; ++r) {
      const float iv = __shfl_sync(0xffffffffu, inv, r);
      if (r < nrows) xn[(size_t)(row0 + r) * 256 + col] = OperandType<TIn>::from_float(x[r] * iv);
    }
  }
}

template <int BN, typename TIn>
__device__ __forceinline__ void epi_act(const GemmArgs& a, const TileCoord& tc, uint32_t taddr, int m, bool valid,
                                        bool tanh_act) {
  TIn* out;
  const float* bias;
  if (a.n_groups == 0) {
    out = static_cast<TIn*>(a.out0) + (size_t)m * a.ld_out + tc.n0;
    bias = a.bias + tc.n0;
  } else {  // mask layer 1: Hm[group][row][col]
    out = static_cast<TIn*>(a.out0) + ((size_t)tc.group * a.M + m) * a.ld_out + tc.n0;
    bias = a.bias + tc.b_row;
  }
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float v[32];
    tmem_ld32(taddr + c * 32, v);
    if (valid) {
      const float4* bp = reinterpret_cast<const float4*>(bias + c * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 bb = bp[q];
        v[4 * q] += bb.x; v[4 * q + 1] += bb.y; v[4 * q + 2] += bb.z; v[4 * q + 3] += bb.w;
      }
#pragma unroll
      for (int i = 0; i < 32; ++i) v[i] = tanh_act ? tanhf(v[i]) : gelu_erf(v[i]);
      store32<TIn>(out + c * 32, v);
    }
  }
}

template <int BN>
__device__ __forceinline__ void epi_glu(const GemmArgs& a, const TileCoord& tc, uint32_t taddr, int m, bool valid) {
  const int g = tc.group;
  const int din = a.g_ncols[g] >> 1;
  float* out = static_cast<float*>(a.out0) + (size_t)m * a.ld_out + a.g_outoff[g];
  const float* bias = a.bias + tc.b_row;
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    if (c * 32 >= tc.n_mma) break;  // uniform over the CTA
    float v[32];
    tmem_ld32(taddr + c * 32, v);
    if (valid) {
      const int col0 = tc.n0 + c * 32;  // interleaved column: (a, g) pairs
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int cc = (col0 >> 1) + i;
        if (cc < din) {
          const float av = v[2 * i] + bias[c * 32 + 2 * i];
          const float gv = v[2 * i + 1] + bias[c * 32 + 2 * i + 1];
          out[cc] = av * sigmoidf_(gv);
        }
      }
    }
  }
}

// ------------------------------------------------------------------------------------------------ kernel
template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kGemmBK * 2;       // 32 KB at BN = 256
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStageOffset = STAGES * kStageBytes;        // epilogue transpose buffers
  static constexpr int kEpiStageBytes = 4 * 32 * 33 * 4;           // 4 warps x [32][33] fp32
  static constexpr int kBarOffset = kStageOffset + kEpiStageBytes;
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
};

template <int BN, int STAGES, int EPI, typename TIn>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ GemmArgs args) {
  using S = GemmSmem<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_b);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x) {
        const TileCoord tc = gemm_decode<BN>(args, tile);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * S::kStageBytes;
          uint8_t* sb = sa + S::kABytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int kx = kb * kGemmBK;
          if (args.a_mode == 0)
            tma_load_2d(sa, &map_a, &full[stage], kx, tc.m0);
          else if (args.a_mode == 1)
            tma_load_3d(sa, &map_a, &full[stage], kx, tc.group, tc.m0);
          else
            tma_load_3d(sa, &map_a, &full[stage], kx, tc.m0, tc.group);
          tma_load_2d(sb, &map_b, &full[stage], kx, tc.b_row);
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {  // drain the copies still in flight before the CTA's shared memory is released
        for (int j = max(0, issued - STAGES); j < issued; ++j) {
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1) && global_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.num_tiles && ok; tile += gridDim.x, ++local) {
        const TileCoord tc = gemm_decode<BN>(args, tile);
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, args.err, kErrWaitMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        const uint32_t idesc = idesc_f16(kGemmBM, tc.n_mma, OperandType<TIn>::kFormat, 0, 0);
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * S::kStageBytes);
          const uint32_t sb = sa + S::kABytes;
#pragma unroll
          for (int kk = 0; kk < kGemmBK / 16; ++kk) {
            const uint64_t ad = sdesc_sw128(sa + kk * 32, 16, 1024);
            const uint64_t bd = sdesc_sw128(sb + kk * 32, 16, 1024);
            mma_f16_ss(d_tmem, ad, bd, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[buf]);
      }
      // all MMAs issued by this thread are complete once `drain` fires
      mma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-5)
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < args.num_tiles; tile += gridDim.x, ++local) {
      const TileCoord tc = gemm_decode<BN>(args, tile);
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if (!mbar_wait_warp(&acc_full[buf], use & 1, args.err, kErrWaitEpilogue, abort_flag)) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(quarter * 32) << 16);
      const int m = tc.m0 + row;
      const bool valid = m < args.M;
      if constexpr (EPI == EPI_QKV) {
        epi_qkv<BN, TIn>(args, tc, taddr, m, valid);
      } else if constexpr (EPI == EPI_RESNORM) {
        float* stage = reinterpret_cast<float*>(smem + S::kStageOffset) + quarter * 32 * 33;
        epi_resnorm<BN, TIn>(args, tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(quarter * 32) << 16),
                             tc.m0 + quarter * 32, lane, stage);
      } else if constexpr (EPI == EPI_GELU) {
        epi_act<BN, TIn>(args, tc, taddr, m, valid, false);
      } else if constexpr (EPI == EPI_MASK_TANH) {
        epi_act<BN, TIn>(args, tc, taddr, m, valid, true);
      } else {
        epi_glu<BN>(args, tc, taddr, m, valid);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

}  // namespace trc
