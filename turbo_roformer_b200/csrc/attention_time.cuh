// Time-mode attention (sequences over the frames of one band and head): the reference's `attention`
// kernel for mode 0 (LoggeL/turbo-roformer src/turbo_roformer/csrc/kernels.cpp:255-388), exact softmax
// with the gate, head merge and scatter to token order, on tcgen05.
//
// A CTA owns three 128-row query tiles of one sequence (an item covers query rows q0 .. q0 + 383) and
// streams 64-key tiles shared by the three:
//   * S = Q K^T (N = 64, both operands in shared memory) lands in TMEM; the tile's softmax warps read the
//     64 scores of their row at once, which frees S for the next key tile's product while the
//     exponentials of this one are computed.
//   * 16-bit P goes to its own TMEM columns and O += P V reads it from there (K = 64); O accumulates in
//     TMEM. Running maximum raised only past 2^8 (O and the row sum then rescaled in place); one key pair
//     in four exponentiated on the FMA pipe (ex2_poly2).
//   * Three query tiles instead of two put three softmax warps on every SM sub-partition (one per
//     tile): the softmax is bound by the latency of its instruction chains, and the third warp hides more
//     of it than the 64-key steps add in per-step work. TMEM: 3 x (S 64 + P 32 + O 64) = 480 columns.
//   * A tile that lies wholly past the sequence's end (the last item of a sequence of 1700 frames
//     holds two tiles) makes no products: its MMA thread still releases the Q buffer and every key
//     stage of the item, after they are filled, so the shared barriers count the same arrivals.
//   * Persistent CTAs; Q double buffered; each item's epilogue (gate / l, store) is deferred to the next
//     item's first step, as in the two-tile kernel.
// Roles (512 threads, four warpgroups): warp 0 TMA, warps 1-3 MMA issuers of tiles 0-2 (warp 1 owns
// TMEM); warps 4-15 softmax + epilogue, warpgroup 1 + x for tile x (thread = query row).
#pragma once

#include "attention.cuh"

namespace trc {

constexpr int kTaTiles = 3;
constexpr int kTaThreads = 512;
// registers per thread after setmaxnreg: warps 0-3 and the softmax warpgroups; the launch gives 128 to
// every thread and 4 * 32 * 56 + 12 * 32 * 152 = 65536 = 512 * 128 (checked before every launch)
constexpr int kTaRegsLow = 56;
constexpr int kTaRegsHigh = 152;
constexpr int kTaKvStages = 6;

struct TaSmem {
  static constexpr int kTileQ = 128 * 64 * 2;  // 16 KB
  static constexpr int kTileKV = 64 * 64 * 2;  // 8 KB
  static constexpr int kQ = 0;                 // [2 buffers][3 tiles]
  static constexpr int kKV = kQ + 2 * kTaTiles * kTileQ;
  static constexpr int kScale = kKV + 2 * kTaKvStages * kTileKV;  // [3 tiles][128] fp32
  static constexpr int kBar = kScale + kTaTiles * 128 * 4;
  static constexpr int kBytes = kBar + 512 + 1024;
  static_assert(kBytes <= 232448, "shared memory per CTA");
};

// TMEM columns: S of tile x at 64 x, O at 192 + 64 x, P (16-bit pairs) at 384 + 32 x
__device__ __forceinline__ uint32_t ta_col_s(int x) { return (uint32_t)x * 64u; }
__device__ __forceinline__ uint32_t ta_col_o(int x) { return 192u + (uint32_t)x * 64u; }
__device__ __forceinline__ uint32_t ta_col_p(int x) { return 384u + (uint32_t)x * 32u; }

template <typename TIn>
__global__ void __launch_bounds__(kTaThreads, 1)
    attention_time_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                      const __grid_constant__ CUtensorMap map_v, const __grid_constant__ AttnArgs args) {
  using S = TaSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars;                  // [2]
  uint64_t* q_empty = q_full + 2;           // [2]
  uint64_t* kv_full = q_empty + 2;          // [stages]
  uint64_t* kv_empty = kv_full + kTaKvStages;
  uint64_t* s_full = kv_empty + kTaKvStages;  // [3]
  uint64_t* s_free = s_full + kTaTiles;
  uint64_t* p_full = s_free + kTaTiles;
  uint64_t* p_free = p_full + kTaTiles;
  uint64_t* o_free = p_free + kTaTiles;
  uint64_t* drain = o_free + kTaTiles;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nsteps = args.n_kv;  // 64-key steps per item

  if (threadIdx.x == 0) {
    for (int b = 0; b < 2; ++b) {
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], kTaTiles);
    }
    for (int x = 0; x < kTaTiles; ++x) {
      mbar_init(&s_full[x], 1);
      mbar_init(&s_free[x], 4);
      mbar_init(&p_full[x], 4);
      mbar_init(&p_free[x], 1);
      mbar_init(&o_free[x], 4);
    }
    for (int s = 0; s < kTaKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], kTaTiles);
    }
    mbar_init(drain, kTaTiles);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kTaRegsLow) : "memory");
    if (warp == 0) {
      // ------------------------------------------------------------------ TMA producer
      if (lane == 0) {
        int kvc = 0, local = 0, q_issued = 0;
        bool ok = true;
        for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x, ++local) {
          const int bh = item / args.q_pairs;
          const int q0 = (item - bh * args.q_pairs) * (128 * kTaTiles);
          const int qb = local & 1;
          if (!mbar_wait(&q_empty[qb], ((uint32_t)(local >> 1) & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&q_full[qb], kTaTiles * S::kTileQ);
          uint8_t* qbuf = smem + S::kQ + qb * kTaTiles * S::kTileQ;
          for (int t = 0; t < kTaTiles; ++t) tma_load_3d(qbuf + t * S::kTileQ, &map_q, &q_full[qb], 0, q0 + 128 * t, bh);
          ++q_issued;
          for (int j = 0; j < nsteps; ++j) {
            const int st = kvc % kTaKvStages;
            const uint32_t u = (uint32_t)(kvc / kTaKvStages);
            if (!mbar_wait(&kv_empty[st], (u & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
              ok = false;
              break;
            }
            uint8_t* kb = smem + S::kKV + st * 2 * S::kTileKV;
            mbar_arrive_expect_tx(&kv_full[st], 2 * S::kTileKV);
            tma_load_3d(kb, &map_k, &kv_full[st], 0, j * 64, bh);
            tma_load_3d(kb + S::kTileKV, &map_v, &kv_full[st], 0, j * 64, bh);
            ++kvc;
          }
        }
        const uint64_t t0 = global_ns();
        for (int k = max(0, kvc - kTaKvStages); k < kvc; ++k)
          while (!mbar_try_wait(&kv_full[k % kTaKvStages], (uint32_t)(k / kTaKvStages) & 1) &&
                 global_ns() - t0 < kWaitLimitNs) {
          }
        for (int k = max(0, q_issued - 2); k < q_issued; ++k)
          while (!mbar_try_wait(&q_full[k & 1], (uint32_t)(k >> 1) & 1) && global_ns() - t0 < kWaitLimitNs) {
          }
      }
    } else {
      // ------------------------------------------------------------------ MMA issuers, one per query tile
      if (lane == 0) {
        const int x = warp - 1;
        const uint32_t idesc_qk = idesc_f16(128, 64, OperandType<TIn>::kFormat, 0, 0);
        const uint32_t idesc_pv = idesc_f16(128, 64, OperandType<TIn>::kFormat, 0, 1);  // V is MN-major
        const uint32_t tS = tmem_base + ta_col_s(x), tP = tmem_base + ta_col_p(x), tO = tmem_base + ta_col_o(x);
        const uint64_t q_desc0 = sdesc_sw128(smem_u32(smem + S::kQ + x * S::kTileQ), 16, 1024);
        const uint64_t k_desc0 = sdesc_sw128(smem_u32(smem + S::kKV), 16, 1024);
        const uint64_t v_desc0 = sdesc_sw128(smem_u32(smem + S::kKV + S::kTileKV), 8192, 1024);
        constexpr uint32_t kStepKV = (2 * S::kTileKV) >> 4;
        constexpr uint32_t kStepQ = (kTaTiles * S::kTileQ) >> 4;
        int kvc = 0, local = 0, active = 0;  // active: items this tile has worked on (o_free phases)
        uint32_t g = 0;
        bool ok = true;
        auto wait = [&](uint64_t* bar, uint32_t parity) {
          if (ok && !mbar_wait(bar, parity, args.err, kErrWaitMma, abort_flag)) ok = false;
          return ok;
        };
        auto issue_s = [&](int j, uint64_t qd, int qb) {
          const int idx = kvc + j;
          const int st = idx % kTaKvStages;
          if (!wait(&kv_full[st], (uint32_t)(idx / kTaKvStages) & 1)) return;
          tc_fence_after();
          const uint64_t kd = k_desc0 + (uint64_t)(st * kStepKV);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) mma_f16_ss(tS, qd + 2 * kk, kd + 2 * kk, idesc_qk, kk > 0 ? 1u : 0u);
          mma_commit(&s_full[x]);
          if (j == nsteps - 1) mma_commit(&q_empty[qb]);
        };
        auto issue_pv = [&](int j) {
          if (!wait(&p_full[x], g & 1u)) return;
          if (j == 0 && active > 0 && !wait(&o_free[x], (uint32_t)(active - 1) & 1)) return;
          tc_fence_after();
          const int st = (kvc + j) % kTaKvStages;
          const uint64_t vd = v_desc0 + (uint64_t)(st * kStepKV);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_f16_ts(tO, tP + kk * 8, vd + kk * (2048 >> 4), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
          mma_commit(&p_free[x]);
          mma_commit(&kv_empty[st]);
        };
        for (int item = blockIdx.x; item < args.num_items && ok; item += gridDim.x, ++local) {
          const int qb = local & 1;
          if (!wait(&q_full[qb], (uint32_t)(local >> 1) & 1)) break;
          const int bh = item / args.q_pairs;
          if ((item - bh * args.q_pairs) * (128 * kTaTiles) + 128 * x >= args.L) {
            // a tile wholly past the sequence's end: no products; release the Q buffer and every key stage
            // of the item once it has been filled (so the arrivals count for this use of each buffer)
            mbar_arrive(&q_empty[qb]);
            for (int j = 0; j < nsteps && ok; ++j) {
              const int idx = kvc + j;
              if (wait(&kv_full[idx % kTaKvStages], (uint32_t)(idx / kTaKvStages) & 1))
                mbar_arrive(&kv_empty[idx % kTaKvStages]);
            }
            kvc += nsteps;
            continue;
          }
          const uint64_t qd = q_desc0 + (uint64_t)(qb * kStepQ);
          if (g > 0 && !wait(&s_free[x], (g - 1) & 1u)) break;
          issue_s(0, qd, qb);
          for (int j = 0; j < nsteps && ok; ++j, ++g) {
            if (j + 1 < nsteps && wait(&s_free[x], g & 1u)) issue_s(j + 1, qd, qb);
            issue_pv(j);
          }
          kvc += nsteps;
          ++active;
        }
        mma_commit(drain);
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitLimitNs) {
        }
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kTaRegsHigh) : "memory");
    // ------------------------------------------------------------------ softmax + epilogue (warps 4-15)
    const int x = (warp - 4) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tS = tmem_base + lane_off + ta_col_s(x);
    const uint32_t tP = tmem_base + lane_off + ta_col_p(x);
    const uint32_t tO = tmem_base + lane_off + ta_col_o(x);
    const float kLog2e = 1.4426950408889634f;
    uint32_t g = 0;
    auto row_token = [&](int item, long* token) -> bool {
      const int bh = item / args.q_pairs;
      const int pos = (item - bh * args.q_pairs) * (128 * kTaTiles) + x * 128 + r;
      if (pos >= args.L || bh >= args.BH) return false;
      const int grp = bh >> 3;
      const int b = grp / args.F, f = grp - b * args.F;
      *token = (((long)b * args.T + pos) * args.F + f) * 8 + (bh & 7);
      return true;
    };
    float* row_scale = reinterpret_cast<float*>(smem + S::kScale) + x * 128 + r;
    auto finish = [&](int prev_item) {
      long th;
      const bool valid = row_token(prev_item, &th);
      const float scale = *row_scale;
      TIn* dst = static_cast<TIn*>(args.O) + th * 64;
#pragma unroll 1
      for (int hc = 0; hc < 2; ++hc) {
        float o[32];
        tmem_ld32(tO + hc * 32, o);
        if (hc == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[x]);
        }
        if (valid) {
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= scale;
          store32<TIn>(dst + hc * 32, o);
        }
      }
    };
    bool alive = true;
    int prev = -1;  // the last item this tile worked on (its epilogue is deferred)
    for (int item = blockIdx.x; item < args.num_items && alive; item += gridDim.x) {
      {
        const int bh = item / args.q_pairs;
        if ((item - bh * args.q_pairs) * (128 * kTaTiles) + 128 * x >= args.L) continue;
      }
      long th0;
      const float gate = row_token(item, &th0) ? args.G[th0] : 0.f;
      float m_run = -INFINITY, l_run = 0.f;
      bool ok = true;
      for (int j = 0; j < nsteps; ++j, ++g) {
        if (!mbar_wait_warp(&s_full[x], g & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float sc[64];
        tmem_ld64(tS, sc);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s_free[x]);
        const int kmax = min(64, args.L - j * 64);
        if (kmax < 64) {
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (i >= kmax) sc[i] = -INFINITY;
        }
        float mx4[4] = {sc[0], sc[1], sc[2], sc[3]};
#pragma unroll
        for (int i = 4; i < 60; i += 8) {
          mx4[0] = fmax3(mx4[0], sc[i], sc[i + 4]);
          mx4[1] = fmax3(mx4[1], sc[i + 1], sc[i + 5]);
          mx4[2] = fmax3(mx4[2], sc[i + 2], sc[i + 6]);
          mx4[3] = fmax3(mx4[3], sc[i + 3], sc[i + 7]);
        }
        const float m_tile =
            fmaxf(fmax3(mx4[0], mx4[1], sc[60]), fmax3(mx4[2], mx4[3], fmax3(sc[61], sc[62], sc[63]))) * kLog2e;
        bool rescale = false;
        float alpha = 1.0f;
        if (j == 0) {
          m_run = m_tile;
        } else {
          const bool need = m_tile > m_run + kRescaleThreshold;
          rescale = __any_sync(0xffffffffu, need);
          if (need) {
            alpha = ex2_approx(m_run - m_tile);
            m_run = m_tile;
          }
        }
        const float2 scale2 = make_float2(kLog2e, kLog2e);
        const float2 shift2 = make_float2(-m_run, -m_run);
        float2 l2 = make_float2(0.f, 0.f);
        auto exp_chunk = [&](int c, uint32_t(&packed)[16]) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int k = c * 32 + i;
            const float2 xv = __ffma2_rn(make_float2(sc[k], sc[k + 1]), scale2, shift2);
            const float2 pv = (i & 7) == 6 ? ex2_poly2(xv) : make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
            l2 = __fadd2_rn(l2, pv);
            packed[i >> 1] = OperandType<TIn>::pack2(pv.x, pv.y);
          }
        };
        {
          uint32_t packed[16];
          exp_chunk(0, packed);
          if (g > 0 && !mbar_wait_warp(&p_free[x], (g - 1) & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (rescale) {
#pragma unroll 1
            for (int h = 0; h < 4; ++h) {
              float o[16];
              uint32_t u[16];
              tmem_ld16(tO + h * 16, o);
#pragma unroll
              for (int i = 0; i < 16; ++i) u[i] = __float_as_uint(o[i] * alpha);
              tmem_st16(tO + h * 16, u);
            }
          }
          tmem_st16(tP, packed);
        }
        {
          uint32_t packed[16];
          exp_chunk(1, packed);
          tmem_st16(tP + 16, packed);
        }
        l_run = l_run * alpha + (l2.x + l2.y);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
        if (j == 0 && prev >= 0) finish(prev);
      }
      if (!ok) {
        alive = false;
        break;
      }
      *row_scale = gate / l_run;
      prev = item;
    }
    if (alive && prev >= 0 && mbar_wait_warp(&p_free[x], (g - 1) & 1u, args.err, kErrWaitSoftmax, abort_flag)) {
      tc_fence_after();
      finish(prev);
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
