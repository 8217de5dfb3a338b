// Fused feed-forward block on tcgen05: X += GELU(xn W1^T + b1) W2^T + b2; xn_out = X / max(|X|, eps).
//
// Replaces the reference's FF pair gemm_gelu + gemm_res_norm (LoggeL/turbo-roformer
// src/turbo_roformer/csrc/kernels.cpp:610-642 and :543-586, sequenced in fast.py:320-333) with one
// kernel in which the hidden activation H never leaves the SM: per 128-row block the 1024 hidden units
// are processed in chunks of 128,
//   G1(c): acc1[c % 2] = xn_block W1[c]^T          (TMEM, 128 x 128 fp32, double buffered)
//   GELU : H = gelu(acc1 + b1[c]) 16-bit, written back over the first half of each 64-column half of
//          acc1[c % 2] (TMEM, the A operand of the next MMA)
//   G2(c): acc2 += H W2[:, c]^T                     (TMEM, 128 x 256, accumulated over the chunks)
// and the residual + norm epilogue of the finished block runs while the next block's chunks are made.
// The 128 x 256 xn block is loaded once per block and stays in shared memory for its eight G1s, so the
// ring of 32 KB stages streams weights only (two W1 k-blocks or one W2 k-block per stage), in the MMA
// order G1(0), G1(1), then G2(c), G1(c + 2) for c = 0..: tcgen05 MMAs of one thread execute in issue
// order, so G1(c + 2) overwrites acc1[c % 2] only after G2(c) has read the H stored there, while the
// GELU warps work on the other buffer. Rows past M are zero-filled by the loads and clipped by the stores.
//
// Roles (448 threads): warp 0 TMA producer, warp 1 MMA issuer + TMEM owner, warps 2-9 GELU (lane
// quarter warp % 4, 64 of the chunk's 128 columns each), warps 10-13 residual + norm (one lane quarter
// each, whole 256-wide rows, so the row norm needs no exchange between warps). Every wait is bounded.
#pragma once

#include "gemm.cuh"
#include "sm100.cuh"

namespace trc {

constexpr int kMlpStages = 3;
constexpr int kMlpBoxes = 4;  // X boxes per epilogue warp
constexpr int kMlpStageBytes = 32 * 1024;
constexpr int kMlpGeluWarps = 8;
constexpr int kMlpEpiWarps = 4;
constexpr int kMlpThreads = 64 + 32 * (kMlpGeluWarps + kMlpEpiWarps);
constexpr int kMlpBoxBytes = 32 * 32 * 4;  // 32 rows x 32 fp32 (or x 64 16-bit) columns

struct MlpArgs {
  int num_blocks;   // 128-row blocks
  int M;            // rows
  int n_chunks;     // hidden / 128
  const float* b1;  // [hidden]
  const float* b2;  // [256]
  float eps;
  int* err;
};

struct MlpSmem {
  static constexpr int kRing = 0;                                  // [stages][32 KB]
  static constexpr int kA = kRing + kMlpStages * kMlpStageBytes;  // [4 k-blocks][128 rows x 64] 16-bit xn block
  static constexpr int kBox = kA + 4 * 16384;                      // [epilogue warp][kMlpBoxes boxes]
  static constexpr int kBar = kBox + kMlpEpiWarps * kMlpBoxes * kMlpBoxBytes;
  static constexpr int kBytes = kBar + 512 + 1024;  // barriers (31 x 8 B + TMEM slot + abort flag), alignment slack
  static_assert(kBytes <= 232448, "shared memory per CTA");
};

// TMEM: acc1 buffers at columns 0 and 128 (H of the chunk in columns +0..31 and +64..95), acc2 at 256..511.
constexpr uint32_t kMlpAcc2 = 256;

template <typename TIn>
__global__ void __launch_bounds__(kMlpThreads, 1)
    mlp_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_w1,
               const __grid_constant__ CUtensorMap map_w2, const __grid_constant__ CUtensorMap map_x,
               const __grid_constant__ CUtensorMap map_xn, const __grid_constant__ MlpArgs args) {
  using S = MlpSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* empty = full + kMlpStages;
  uint64_t* a1_full = empty + kMlpStages;  // [2] G1 chunk in acc1 (MMA commit)
  uint64_t* h_full = a1_full + 2;          // [2] H chunk written to TMEM (one arrive per GELU warp)
  uint64_t* a_full = h_full + 2;           // xn block loaded (TMA bytes)
  uint64_t* a_empty = a_full + 1;          // the block's last G1 has read the xn block (MMA commit)
  uint64_t* a2_full = a_empty + 1;         // block's acc2 complete (MMA commit)
  uint64_t* a2_empty = a2_full + 1;        // epilogue done with acc2 (one arrive per epilogue warp)
  uint64_t* xbars = a2_empty + 1;          // [epilogue warp][kMlpBoxes] X box loads
  uint64_t* drain = xbars + kMlpBoxes * kMlpEpiWarps;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nch = args.n_chunks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kMlpStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&a1_full[b], 1);
      mbar_init(&h_full[b], kMlpGeluWarps);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    mbar_init(a2_full, 1);
    mbar_init(a2_empty, kMlpEpiWarps);
    for (int b = 0; b < kMlpBoxes * kMlpEpiWarps; ++b) mbar_init(&xbars[b], 1);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_a);
    tma_prefetch_desc(&map_w1);
    tma_prefetch_desc(&map_w2);
    tma_prefetch_desc(&map_x);
    tma_prefetch_desc(&map_xn);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0, issued = 0;
      uint32_t phase = 0;
      bool ok = true;
      auto next_stage = [&](int bytes) -> uint8_t* {
        if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrWaitProducer, abort_flag)) {
          ok = false;
          return nullptr;
        }
        mbar_arrive_expect_tx(&full[stage], bytes);
        return smem + S::kRing + stage * kMlpStageBytes;
      };
      auto advance = [&]() {
        ++issued;
        if (++stage == kMlpStages) {
          stage = 0;
          phase ^= 1;
        }
      };
      int a_loads = 0;
      for (int blk = blockIdx.x; blk < args.num_blocks && ok; blk += gridDim.x) {
        const int m0 = blk * 128;
        // the xn block: once the previous block's last G1 has read the buffer
        if (a_loads > 0 && !mbar_wait(a_empty, (uint32_t)(a_loads - 1) & 1, args.err, kErrWaitProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(a_full, 4 * 16384);
        for (int kb = 0; kb < 4; ++kb) tma_load_2d(smem + S::kA + kb * 16384, &map_a, a_full, kb * 64, m0);
        ++a_loads;
        auto load_g1 = [&](int c) {  // 2 stages of 2 k-blocks: W1[c*128.., k] (16 KB each)
          for (int s = 0; s < 2 && ok; ++s) {
            uint8_t* st = next_stage(kMlpStageBytes);
            if (!st) return;
            tma_load_2d(st, &map_w1, &full[stage], (2 * s) * 64, c * 128);
            tma_load_2d(st + 16384, &map_w1, &full[stage], (2 * s + 1) * 64, c * 128);
            advance();
          }
        };
        auto load_g2 = [&](int c) {  // 2 k-blocks: W2[0..256, c*128 + kb*64..] (32 KB)
          for (int kb = 0; kb < 2 && ok; ++kb) {
            uint8_t* st = next_stage(kMlpStageBytes);
            if (!st) return;
            tma_load_2d(st, &map_w2, &full[stage], c * 128 + kb * 64, 0);
            advance();
          }
        };
        load_g1(0);
        if (nch > 1) load_g1(1);
        for (int c = 0; c < nch && ok; ++c) {
          load_g2(c);
          if (c + 2 < nch) load_g1(c + 2);
        }
      }
      if (!ok) {  // drain the copies still in flight before the CTA's shared memory is released
        const uint64_t t0 = global_ns();
        for (int j = max(0, issued - kMlpStages); j < issued; ++j)
          while (!mbar_try_wait(&full[j % kMlpStages], (j / kMlpStages) & 1) && global_ns() - t0 < kWaitLimitNs) {
          }
        if (a_loads > 0)
          while (!mbar_try_wait(a_full, (uint32_t)(a_loads - 1) & 1) && global_ns() - t0 < kWaitLimitNs) {
          }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc1 = idesc_f16(128, 128, OperandType<TIn>::kFormat, 0, 0);
      const uint32_t idesc2 = idesc_f16(128, 256, OperandType<TIn>::kFormat, 0, 0);
      const uint32_t abase = smem_u32(smem + S::kA);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t gch = 0;  // chunks of all blocks before this block (acc1 / H buffer = chunk parity)
      int lb = 0;        // blocks of this CTA so far (a2 phases)
      bool ok = true;
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        if (ok && !mbar_wait(bar, parity, args.err, kErrWaitMma, abort_flag)) ok = false;
        return ok;
      };
      auto take_stage = [&]() -> uint32_t {
        if (!wait(&full[stage], phase)) return 0;
        tc_fence_after();
        return smem_u32(smem + S::kRing + stage * kMlpStageBytes);
      };
      auto release_stage = [&]() {
        mma_commit(&empty[stage]);
        if (++stage == kMlpStages) {
          stage = 0;
          phase ^= 1;
        }
      };
      // G1(c) into acc1[chunk parity]; the buffer's previous reader (G2 of the chunk two before) was
      // issued earlier by this thread, and the tensor core runs MMAs in issue order
      auto g1 = [&](int c) {
        const uint32_t b = (gch + c) & 1;
        for (int s = 0; s < 2 && ok; ++s) {
          const uint32_t st = take_stage();
          if (!ok) return;
#pragma unroll
          for (int kb = 0; kb < 2; ++kb)
#pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              mma_f16_ss(tmem_base + b * 128, sdesc_sw128(abase + (2 * s + kb) * 16384 + kk * 32, 16, 1024),
                         sdesc_sw128(st + kb * 16384 + kk * 32, 16, 1024), idesc1, (s | kb | kk) != 0 ? 1u : 0u);
          release_stage();
        }
        mma_commit(&a1_full[b]);
        if (c == nch - 1) mma_commit(a_empty);
      };
      // G2(c): A = H in TMEM (k 0..63 at columns +0..31, k 64..127 at +64..95 of acc1[chunk parity])
      auto g2 = [&](int c) {
        const uint32_t b = (gch + c) & 1;
        for (int s = 0; s < 2 && ok; ++s) {
          const uint32_t st = take_stage();
          if (!ok) return;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ts(tmem_base + kMlpAcc2, tmem_base + b * 128 + s * 64 + kk * 8, sdesc_sw128(st + kk * 32, 16, 1024),
                       idesc2, (c | s | kk) != 0 ? 1u : 0u);
          release_stage();
        }
      };
      for (int blk = blockIdx.x; blk < args.num_blocks && ok; blk += gridDim.x, ++lb) {
        if (!wait(a_full, (uint32_t)lb & 1)) break;
        tc_fence_after();
        g1(0);
        if (nch > 1) g1(1);
        for (int c = 0; c < nch && ok; ++c) {
          const uint32_t gc = gch + c;
          if (!wait(&h_full[gc & 1], (gc >> 1) & 1)) break;
          if (c == 0 && lb > 0 && !wait(a2_empty, (uint32_t)(lb - 1) & 1)) break;
          tc_fence_after();
          g2(c);
          if (c + 2 < nch) g1(c + 2);
        }
        if (!ok) break;
        mma_commit(a2_full);
        gch += nch;
      }
      mma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else if (warp < 2 + kMlpGeluWarps) {
    // ------------------------------------------------------------------ GELU warps
    const int gw = warp - 2;
    const int quarter = warp & 3;
    const int half = gw >> 2;  // columns [64 half, 64 half + 64) of the chunk
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    uint32_t gc = 0;
    bool ok = true;
    for (int blk = blockIdx.x; blk < args.num_blocks && ok; blk += gridDim.x) {
      for (int c = 0; c < nch; ++c, ++gc) {
        const uint32_t b = gc & 1;
        if (!mbar_wait_warp(&a1_full[b], (gc >> 1) & 1, args.err, kErrWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v0[32], v1[32];
        const uint32_t ta = tmem_base + lane_off + b * 128 + half * 64;
        tmem_ld32(ta, v0);
        tmem_ld32(ta + 32, v1);
        const float4* bp = reinterpret_cast<const float4*>(args.b1 + c * 128 + half * 64);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b0 = __ldg(bp + q), b1 = __ldg(bp + 8 + q);
          v0[4 * q] += b0.x; v0[4 * q + 1] += b0.y; v0[4 * q + 2] += b0.z; v0[4 * q + 3] += b0.w;
          v1[4 * q] += b1.x; v1[4 * q + 1] += b1.y; v1[4 * q + 2] += b1.z; v1[4 * q + 3] += b1.w;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float2 g0 = gelu_erf2(make_float2(v0[i], v0[i + 1]));
          const float2 g1 = gelu_erf2(make_float2(v1[i], v1[i + 1]));
          v0[i] = g0.x; v0[i + 1] = g0.y;
          v1[i] = g1.x; v1[i + 1] = g1.y;
        }
        // H over this warp's own (already loaded) columns: 64 16-bit values in 32 columns
        uint32_t p0[16], p1[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          p0[i] = OperandType<TIn>::pack2(v0[2 * i], v0[2 * i + 1]);
          p1[i] = OperandType<TIn>::pack2(v1[2 * i], v1[2 * i + 1]);
        }
        tmem_st16(ta, p0);
        tmem_st16(ta + 16, p1);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&h_full[b]);
      }
    }
  } else {
    // ------------------------------------------------------------------ residual + norm (warps 10-13)
    const int ew = warp - 2 - kMlpGeluWarps;
    const int quarter = warp & 3;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t t2 = tmem_base + lane_off + kMlpAcc2;
    uint8_t* box = smem + S::kBox + ew * kMlpBoxes * kMlpBoxBytes;
    uint64_t* xb = xbars + ew * kMlpBoxes;
    int pend[kMlpBoxes];  // lane 0: parity of the X load in flight per box, -1 if none
    for (int k = 0; k < kMlpBoxes; ++k) pend[k] = -1;
    const int swz = lane & 7;
    auto load_x = [&](int k, int col, int row0, int parity) {
      mbar_arrive_expect_tx(&xb[k], kMlpBoxBytes);
      tma_load_2d(box + k * kMlpBoxBytes, &map_x, &xb[k], col, row0);
      pend[k] = parity;
    };
    int lb = 0;
    for (int blk = blockIdx.x; blk < args.num_blocks; blk += gridDim.x, ++lb) {
      const int row0 = blk * 128 + quarter * 32;
      const bool live = row0 < args.M;  // a warp whose rows all lie past M moves no data
      if (live && lane == 0) {
        bulk_wait_read<0>();  // the previous block's stores have read the boxes
        for (int k = 0; k < kMlpBoxes; ++k) load_x(k, k * 32, row0, 0);  // X chunks 0..3, ahead of acc2
      }
      if (!mbar_wait_warp(a2_full, (uint32_t)lb & 1, args.err, kErrWaitEpilogue, abort_flag)) break;
      tc_fence_after();
      bool ok = true;
      float ss = 0.f;
      // pass 1: X_new = X + acc2 + b2, 32 columns at a time, kept in TMEM and stored to X by TMA
#pragma unroll 1
      for (int c = 0; c < 8 && live; ++c) {
        const int k = c % kMlpBoxes;
        if (!mbar_wait_warp(&xb[k], (uint32_t)(c / kMlpBoxes) & 1, args.err, kErrWaitEpilogue, abort_flag)) {
          ok = false;
          break;
        }
        if (lane == 0) pend[k] = -1;
        float v[32];
        tmem_ld32(t2 + c * 32, v);
        uint8_t* rowp = box + k * kMlpBoxBytes + lane * 128;
        const float4* bp = reinterpret_cast<const float4*>(args.b2 + c * 32);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 x4 = *reinterpret_cast<const float4*>(rowp + ((j ^ swz) << 4));
          const float4 b4 = __ldg(bp + j);
          v[4 * j] += x4.x + b4.x;
          v[4 * j + 1] += x4.y + b4.y;
          v[4 * j + 2] += x4.z + b4.z;
          v[4 * j + 3] += x4.w + b4.w;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) ss = fmaf(v[i], v[i], ss);
        tmem_st32(t2 + c * 32, v);
#pragma unroll
        for (int j = 0; j < 8; ++j)
          *reinterpret_cast<float4*>(rowp + ((j ^ swz) << 4)) =
              make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        fence_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_store_2d(&map_x, box + k * kMlpBoxBytes, c * 32, row0);
          bulk_commit();
          // refill the box stored one chunk earlier (its store has had a chunk's time to read it) with
          // the chunk kMlpBoxes after it; waiting on this chunk's own store would stall every chunk
          const int cp = c - 1;
          if (cp >= 0 && cp + kMlpBoxes < 8) {
            bulk_wait_read<1>();
            load_x(cp % kMlpBoxes, (cp + kMlpBoxes) * 32, row0, 1);
          }
        }
      }
      if (!ok) break;
      tmem_wait_st();
      if (live) {
        // pass 2: xn = X_new / max(|X_new|, eps), 16-bit, 64 columns per box
        const float inv = 1.0f / fmaxf(sqrtf(ss), args.eps);
        if (lane == 0) bulk_wait_read<0>();  // every box's X store has read it
        __syncwarp();
#pragma unroll 1
        for (int k4 = 0; k4 < 4; ++k4) {
          const int k = k4;
          uint8_t* rowp = box + k * kMlpBoxBytes + lane * 128;
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float v[32];
            tmem_ld32(t2 + k4 * 64 + h * 32, v);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              uint4 q;
              q.x = OperandType<TIn>::pack2(v[8 * t] * inv, v[8 * t + 1] * inv);
              q.y = OperandType<TIn>::pack2(v[8 * t + 2] * inv, v[8 * t + 3] * inv);
              q.z = OperandType<TIn>::pack2(v[8 * t + 4] * inv, v[8 * t + 5] * inv);
              q.w = OperandType<TIn>::pack2(v[8 * t + 6] * inv, v[8 * t + 7] * inv);
              *reinterpret_cast<uint4*>(rowp + (((h * 4 + t) ^ swz) << 4)) = q;
            }
          }
          fence_async_smem();
          __syncwarp();
          if (lane == 0) {
            tma_store_2d(&map_xn, box + k * kMlpBoxBytes, k4 * 64, row0);
            bulk_commit();
          }
        }
      }
      // acc2 (and the X_new kept in it) has been read: the next block's G2 may start
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(a2_empty);
    }
    if (lane == 0) {
      const uint64_t t0 = global_ns();
      for (int k = 0; k < kMlpBoxes; ++k)
        if (pend[k] >= 0)
          while (!mbar_try_wait(&xb[k], (uint32_t)pend[k]) && global_ns() - t0 < kWaitLimitNs) {
          }
      bulk_wait<0>();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace trc
