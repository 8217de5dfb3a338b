// Exact-softmax gated attention on tcgen05 (flash-style, online softmax with exact rescaling).
//
// Replaces the reference's AVX-512 `attention` kernel (LoggeL/turbo-roformer
// src/turbo_roformer/csrc/kernels.cpp:255-388): per (sequence, head) S = Q K^T (scale folded into W_q),
// softmax over the keys, O = P V, then x sigmoid gate, head merge and scatter back to token order.
// The reference keeps whole score rows (two passes); here one CTA owns 128 query rows and streams
// 128-key tiles: S and the PV partial product live in TMEM, unnormalised P (16-bit) is staged in
// shared memory in the 128-byte-swizzled K-major layout the tensor core reads.
//
// Layout: Q, K, V are [BH, L, 64] 16-bit, row-major, unpadded; the 3-D TMA maps zero-fill rows >= L.
//   time mode (mode 0): sequences = (batch, band, head), L = T frames, one sequence per CTA tile.
//   freq mode (mode 1): sequences = (batch, frame, head), L = bands <= 64, two sequences per 128-row
//                       tile with a block-diagonal mask.
// Roles (192 threads): warp 0 TMA, warp 1 MMA issuer + TMEM owner, warps 2-5 softmax + epilogue
// (thread = query row).
#pragma once

#include "gemm.cuh"  // store32
#include "sm100.cuh"

namespace trc {

constexpr int kAttnThreads = 192;
constexpr int kAttnKvStages = 3;

struct AttnArgs {
  int num_tiles;
  int q_tiles;  // query tiles per sequence (time) ; 1 (freq)
  int n_kv;     // key tiles per sequence (time) ; 1 (freq)
  int L;        // valid length of every sequence
  int BH;       // number of sequences
  int mode;     // 0 time, 1 freq
  int T, F;     // frames, bands (per batch item)
  const float* G;  // gates [tokens][8]
  void* O;         // [tokens][512] 16-bit
  int* err;
};

struct AttnSmem {
  static constexpr int kTile = 128 * 64 * 2;  // 16 KB: 128 rows x 64 dims
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kTile;
  static constexpr int kV = kK + kAttnKvStages * kTile;
  static constexpr int kP = kV + kAttnKvStages * kTile;  // 2 swizzle atoms along keys: 32 KB
  static constexpr int kBar = kP + 2 * kTile;
  static constexpr int kBytes = kBar + 256 + 1024;
};

template <typename TIn>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attention_kernel(const __grid_constant__ CUtensorMap map_q, const __grid_constant__ CUtensorMap map_k,
                     const __grid_constant__ CUtensorMap map_v, const __grid_constant__ AttnArgs args) {
  using S = AttnSmem;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + S::kBar);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;
  uint64_t* v_full = k_full + kAttnKvStages;
  uint64_t* kv_empty = v_full + kAttnKvStages;
  uint64_t* s_full = kv_empty + kAttnKvStages;  // [2]
  uint64_t* s_empty = s_full + 2;               // [2]
  uint64_t* p_full = s_empty + 2;
  uint64_t* pv_full = p_full + 1;
  uint64_t* pv_empty = pv_full + 1;
  uint64_t* drain = pv_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tile = blockIdx.x;
  const bool freq = args.mode == 1;
  int bh0, q0;
  if (freq) {
    bh0 = 2 * tile;
    q0 = 0;
  } else {
    bh0 = tile / args.q_tiles;
    q0 = (tile - bh0 * args.q_tiles) * 128;
  }
  const int n_kv = args.n_kv;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttnKvStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&s_empty[b], 128);
    }
    mbar_init(p_full, 128);
    mbar_init(pv_full, 1);
    mbar_init(pv_empty, 128);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&map_q);
    tma_prefetch_desc(&map_k);
    tma_prefetch_desc(&map_v);
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);  // S0 [0,128), S1 [128,256), PV [256,320)
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, S::kTile);
      tma_load_3d(smem + S::kQ, &map_q, q_full, 0, q0, bh0);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % kAttnKvStages;
        const uint32_t u = (uint32_t)(j / kAttnKvStages);
        if (!mbar_wait(&kv_empty[st], (u & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&k_full[st], S::kTile);
        tma_load_3d(smem + S::kK + st * S::kTile, &map_k, &k_full[st], 0, j * 128, bh0);
        mbar_arrive_expect_tx(&v_full[st], S::kTile);
        tma_load_3d(smem + S::kV + st * S::kTile, &map_v, &v_full[st], 0, j * 128, bh0);
        ++issued;
      }
      {  // drain: wait (bounded) until every issued copy has landed before the CTA may exit
        const uint64_t t0 = global_ns();
        while (!mbar_try_wait(q_full, 0) && global_ns() - t0 < kWaitLimitNs) {
        }
        if (!ok) {
          for (int j = max(0, issued - kAttnKvStages); j < issued; ++j) {
            const int st = j % kAttnKvStages;
            const uint32_t ph = (uint32_t)(j / kAttnKvStages) & 1;
            const uint64_t t1 = global_ns();
            while (!(mbar_try_wait(&k_full[st], ph) && mbar_try_wait(&v_full[st], ph)) &&
                   global_ns() - t1 < kWaitLimitNs) {
            }
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc_qk = idesc_f16(128, 128, OperandType<TIn>::kFormat, 0, 0);
      const uint32_t idesc_pv = idesc_f16(128, 64, OperandType<TIn>::kFormat, 0, 1);  // V is MN-major
      const uint32_t sq = smem_u32(smem + S::kQ);
      const uint32_t sp = smem_u32(smem + S::kP);
      bool ok = mbar_wait(q_full, 0, args.err, kErrWaitMma, abort_flag);
      auto issue_pv = [&](int i) -> bool {
        const int st = i % kAttnKvStages;
        const uint32_t u = (uint32_t)(i / kAttnKvStages);
        if (!mbar_wait(p_full, (uint32_t)i & 1, args.err, kErrWaitMma, abort_flag)) return false;
        if (!mbar_wait(&v_full[st], u & 1, args.err, kErrWaitMma, abort_flag)) return false;
        if (!mbar_wait(pv_empty, ((uint32_t)i & 1) ^ 1, args.err, kErrWaitMma, abort_flag)) return false;
        tc_fence_after();
        const uint32_t sv = smem_u32(smem + S::kV + st * S::kTile);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {  // 16 keys per MMA
          const uint64_t ad = sdesc_sw128(sp + (kk >> 2) * S::kTile + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sv + kk * 2048, 8192, 1024);
          mma_f16_ss(tmem_base + 256, ad, bd, idesc_pv, kk > 0 ? 1u : 0u);
        }
        mma_commit(pv_full);
        mma_commit(&kv_empty[st]);
        return true;
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j % kAttnKvStages;
        const uint32_t u = (uint32_t)(j / kAttnKvStages);
        const int sb = j & 1;
        if (!mbar_wait(&k_full[st], u & 1, args.err, kErrWaitMma, abort_flag) ||
            !mbar_wait(&s_empty[sb], (((uint32_t)j >> 1) & 1) ^ 1, args.err, kErrWaitMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + S::kK + st * S::kTile);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const uint64_t ad = sdesc_sw128(sq + kk * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(sk + kk * 32, 16, 1024);
          mma_f16_ss(tmem_base + (uint32_t)(sb * 128), ad, bd, idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(&s_full[sb]);
        if (j > 0 && !issue_pv(j - 1)) ok = false;
      }
      if (ok && n_kv > 0) issue_pv(n_kv - 1);
      mma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax + epilogue (warps 2-5)
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int seq = freq ? bh0 + (r >> 6) : bh0;
    const int pos = freq ? (r & 63) : q0 + r;
    const int my_block = r >> 6;  // freq: which of the two sequences
    const float kLog2e = 1.4426950408889634f;
    float o[64];
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;
    uint8_t* prow = smem + S::kP + r * 128;
    bool ok = true;

    for (int j = 0; j < n_kv; ++j) {
      const int sb = j & 1;
      if (!mbar_wait_warp(&s_full[sb], ((uint32_t)j >> 1) & 1, args.err, kErrWaitSoftmax, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t s_addr = tmem_base + lane_off + (uint32_t)(sb * 128);
      const int key0 = j * 128;
      // pass 1: row maximum over the valid keys
      float mx = -INFINITY;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(s_addr + c * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kc = c * 32 + i;
          const bool kv = freq ? ((kc >> 6) == my_block && (kc & 63) < args.L) : (key0 + kc < args.L);
          if (kv) mx = fmaxf(mx, v[i]);
        }
      }
      const float m_new = fmaxf(m_run, mx * kLog2e);
      // fold in the previous tile's P V (computed relative to m_run)
      if (j > 0) {
        if (!mbar_wait_warp(pv_full, (uint32_t)(j - 1) & 1, args.err, kErrWaitSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem_base + lane_off + 256, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] += v[i];
        tmem_ld32(tmem_base + lane_off + 256 + 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 + i] += v[i];
        tc_fence_before();
        mbar_arrive(pv_empty);
      }
      const float alpha = ex2_approx(m_run - m_new);  // 0 on the first tile (m_run = -inf)
#pragma unroll
      for (int i = 0; i < 64; ++i) o[i] *= alpha;
      l_run *= alpha;
      m_run = m_new;
      // pass 2: P = 2^(s log2e - m), 16-bit, into the swizzled K-major P tile
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        float v[32];
        tmem_ld32(s_addr + c * 32, v);
        uint32_t packed[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          float p2[2];
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int kc = c * 32 + i + e;
            const bool kv = freq ? ((kc >> 6) == my_block && (kc & 63) < args.L) : (key0 + kc < args.L);
            p2[e] = kv ? ex2_approx(fmaf(v[i + e], kLog2e, -m_run)) : 0.f;
            l_run += p2[e];
          }
          packed[i >> 1] = OperandType<TIn>::pack2(p2[0], p2[1]);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int chunk = c * 4 + q;  // 16-byte chunk (8 keys) within the 256-byte row
          const int atom = chunk >> 3, cc = chunk & 7;
          uint4* dst = reinterpret_cast<uint4*>(prow + atom * S::kTile + ((cc ^ (r & 7)) << 4));
          *dst = make_uint4(packed[4 * q], packed[4 * q + 1], packed[4 * q + 2], packed[4 * q + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(&s_empty[sb]);
      fence_async_smem();
      mbar_arrive(p_full);
    }
    if (ok && n_kv > 0) {
      if (mbar_wait_warp(pv_full, (uint32_t)(n_kv - 1) & 1, args.err, kErrWaitSoftmax, abort_flag)) {
        tc_fence_after();
        float v[32];
        tmem_ld32(tmem_base + lane_off + 256, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] += v[i];
        tmem_ld32(tmem_base + lane_off + 256 + 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 + i] += v[i];
        // epilogue: out = o / l * gate -> O[token][h*64 + d]
        const bool valid = pos < args.L && seq < args.BH;
        if (valid) {
          const int h = seq & 7;
          const int grp = seq >> 3;
          long token;
          if (!freq) {  // grp = b*F + f, pos = t
            const int b = grp / args.F, f = grp - b * args.F;
            token = ((long)b * args.T + pos) * args.F + f;
          } else {  // grp = b*T + t, pos = f
            token = (long)grp * args.F + pos;
          }
          const float scale = args.G[token * 8 + h] / l_run;
          TIn* dst = static_cast<TIn*>(args.O) + token * 512 + h * 64;
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = o[i] * scale;
          store32<TIn>(dst, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = o[32 + i] * scale;
          store32<TIn>(dst + 32, v);
        }
      }
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
