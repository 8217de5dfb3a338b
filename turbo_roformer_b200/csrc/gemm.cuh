// Persistent tcgen05 GEMM  D[128 x BN] = A[128 x K] * B[BN x K]^T  with fused epilogues.
//
// Roles (320 threads): warp 0 = TMA producer, warp 1 = MMA issuer + TMEM owner, warps 2-9 = epilogue.
// A and B are K-major 16-bit tiles (128-byte swizzle) streamed through a STAGES-deep shared-memory ring;
// the accumulator lives in TMEM, double buffered (2 x BN columns) so the epilogue of tile i overlaps the
// MMAs of tile i+1. Epilogue warp w reads TMEM lane quarter (w % 4) and one half of the columns, so
// two warps share each SM sub-partition. 16-bit outputs are written through 128-byte-swizzled shared
// staging slabs (128 rows x 64 columns) and stored with TMA, so global writes are whole lines and
// asynchronous; the fp32 residual stream is updated by warp-cooperative coalesced row segments.
//
// Epilogues (the reference kernels they replace, LoggeL/turbo-roformer src/turbo_roformer/csrc/kernels.cpp):
//   EPI_QKV       qkv_rope_gemm (:442-540): rotary on q,k in fp32, Q/K/V stored per head as TMA boxes of
//                 the attention layout, sigmoid gates (16-column tile)
//   EPI_RESNORM   gemm_res_norm (:543-586): X += acc (+ bias); xn = X / max(|X|, eps)
//   EPI_GELU      gemm_gelu (:610-642):     H = gelu(acc + b), erf by A&S 7.1.28
//   EPI_MASK_TANH mask MLP layer 1 (fast.py:354):  tanh(acc + b1) per band
//   EPI_MASK_GLU  mask MLP layer 2 + GLU (fast.py:355-357): a * sigmoid(g), with (a, g) rows interleaved
//   EPI_BAND      band split (model.py:147-155): X = acc + b per band, and the transformers' first norm
//                 xn = X / max(|X|, eps) (kernels.cpp:102-137) in the same pass
//   EPI_F32       Y = acc + b in fp32 (2-D, or 3-D per group): the unfused residual branch for models whose
//                 width is not 256 (the norm then runs as add_rmsnorm / rownorm)
//   EPI_QKVS      EPI_QKV with the A tile streamed with B (K other than 256: the resident tile would not fit)
#pragma once

#include "sm100.cuh"

namespace trc {

enum EpiKind : int {
  EPI_QKV = 0, EPI_RESNORM = 1, EPI_GELU = 2, EPI_MASK_TANH = 3, EPI_MASK_GLU = 4, EPI_BAND = 5, EPI_F32 = 6,
  EPI_QKVS = 7
};
__host__ __device__ constexpr bool is_qkv(int epi) { return epi == EPI_QKV || epi == EPI_QKVS; }

// How a tile's 128 A rows are addressed.
enum AMode : int {
  A_ROWS = 0,        // 2-D [rows][K]: 128 consecutive rows
  A_GROUP_ROWS = 1,  // 3-D (K, group, rows): rows of one group (mask layer 1: one band of every frame)
  A_ROWS_GROUP = 2,  // 3-D (K, rows, group): group-major storage (mask layer 2)
  A_TIME_SEQ = 3,    // 4-D (K, band, frame, batch): 128 consecutive frames of one band (time qkv)
  A_FREQ_PAIR = 4,   // 3-D (K, band, frame): two frames x 64 band slots (freq qkv)
  A_BAND = 5,        // 2-D [rows][K]: each group (band) reads its own K range (g_koff, g_kblocks)
};

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;
constexpr int kEpiWarps = 8;
constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kMaxGroups = 64;
constexpr int kSlabBytes = 128 * 128;  // 128 rows x 64 16-bit columns

struct GemmArgs {
  // ---- schedule
  int num_tiles;
  int k_blocks;   // K / 64
  int a_mode;     // AMode
  int M;          // valid rows: rows (dense), rows per group (grouped), T (time qkv), B*T (freq qkv)
  int n_tiles;    // N tiles per M tile (dense and qkv)
  int N;          // valid columns (dense and qkv)
  int m_tiles;    // time qkv: M tiles per (batch, band)
  int F;          // bands (qkv)
  int T;          // frames per chunk (qkv)
  int n_groups;   // grouped GEMMs: number of groups (0 otherwise)
  int g_tile_start[kMaxGroups + 1];
  int g_ntiles[kMaxGroups];
  int g_brow[kMaxGroups];    // first B row of the group
  int g_ncols[kMaxGroups];   // valid columns of the group
  int g_outoff[kMaxGroups];  // output column offset of the group (mask GLU)
  int g_koff[kMaxGroups];    // A_BAND: first K element of the group (a multiple of 64)
  int g_kblocks[kMaxGroups]; // A_BAND: K blocks of the group
  // ---- epilogue
  void* out0;
  void* out1;
  void* out2;
  void* out3;
  const float* bias;   // indexed by B row (nullptr = none)
  int bias_gstride;    // EPI_F32: bias of group g starts at bias + g * bias_gstride
  const float* bias2;  // qkv: gate bias [8]
  const float* cos_tab;
  const float* sin_tab;
  int ld_out;
  float eps;
  int* err;
};

struct TileCoord {
  int m0, n0, group, b_row, n_valid, n_mma;
  int koff, kblocks;  // K range: [koff, koff + 64 * kblocks)
  int a1, a2, a3;  // TMA coordinates of A after the K coordinate
  int b, f;        // time qkv: batch item and band of the tile
};

template <int BN>
__device__ __forceinline__ TileCoord gemm_decode(const GemmArgs& a, int tile) {
  TileCoord c;
  c.group = 0;
  c.b = 0;
  c.f = 0;
  c.a3 = 0;
  c.koff = 0;
  c.kblocks = a.k_blocks;
  int nt;
  if (a.n_groups > 0) {
    int g = 0;
    while (g + 1 < a.n_groups && tile >= a.g_tile_start[g + 1]) ++g;
    const int local = tile - a.g_tile_start[g];
    const int mt = local / a.g_ntiles[g];
    nt = local - mt * a.g_ntiles[g];
    c.group = g;
    c.m0 = mt * kGemmBM;
    c.n0 = nt * BN;
    c.b_row = a.g_brow[g] + c.n0;
    c.n_valid = min(BN, a.g_ncols[g] - c.n0);
    if (a.a_mode == A_BAND) {
      c.a1 = c.m0;
      c.a2 = 0;
      c.koff = a.g_koff[g];
      c.kblocks = a.g_kblocks[g];
    } else if (a.a_mode == A_GROUP_ROWS) {
      c.a1 = g;
      c.a2 = c.m0;
    } else {
      c.a1 = c.m0;
      c.a2 = g;
    }
  } else if (a.a_mode == A_TIME_SEQ) {
    const int per = a.m_tiles * a.n_tiles;
    const int bf = tile / per;
    const int rem = tile - bf * per;
    const int mt = rem / a.n_tiles;
    nt = rem - mt * a.n_tiles;
    c.b = bf / a.F;
    c.f = bf - c.b * a.F;
    c.m0 = mt * kGemmBM;  // first frame
    c.n0 = nt * BN;
    c.b_row = c.n0;
    c.n_valid = min(BN, a.N - c.n0);
    c.a1 = c.f;
    c.a2 = c.m0;
    c.a3 = c.b;
  } else {
    const int mt = tile / a.n_tiles;
    nt = tile - mt * a.n_tiles;
    c.m0 = a.a_mode == A_FREQ_PAIR ? 2 * mt : mt * kGemmBM;  // freq: first frame of the pair
    c.n0 = nt * BN;
    c.b_row = c.n0;
    c.n_valid = min(BN, a.N - c.n0);
    if (a.a_mode == A_FREQ_PAIR) {
      c.a1 = 0;
      c.a2 = c.m0;
    } else {
      c.a1 = c.m0;
      c.a2 = 0;
    }
  }
  c.n_mma = (c.n_valid + 15) & ~15;
  return c;
}

__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + __expf(-x)); }
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// tanh(x) = 1 - 2 / (e^(2x) + 1) with the MUFU exponential and reciprocal: absolute error ~1e-7 over the
// whole range (saturates cleanly to +-1), against a relative 2^-11 from rounding the result to 16 bits.
__device__ __forceinline__ float tanh_exp(float x) {
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(x * 2.8853900817779268f));  // 2 log2(e)
  return fmaf(-2.0f, rcp_approx(e + 1.0f), 1.0f);
}

// Exact-form GELU 0.5·x·(1 + erf(x/√2)) on a pair of values. erf(z), z >= 0, is Abramowitz & Stegun 7.1.28:
// 1 - (1 + a1·z + ... + a6·z^6)^-16 (|error| <= 3e-7), one reciprocal per value and the polynomial in packed
// fp32 pairs. The odd extension folds into 0.5·x + 0.5·|x|·erf(|x|/√2). The reference's CPU epilogue also
// evaluates erf by an Abramowitz & Stegun rational form (kernels.cpp:588-607, formula 7.1.26).
__device__ __forceinline__ float2 gelu_erf2(float2 x) {
  const float2 ax = make_float2(fabsf(x.x), fabsf(x.y));
  const float2 z = __fmul2_rn(ax, make_float2(0.70710678118654752f, 0.70710678118654752f));
  float2 p = __ffma2_rn(make_float2(4.30638e-5f, 4.30638e-5f), z, make_float2(2.765672e-4f, 2.765672e-4f));
  p = __ffma2_rn(p, z, make_float2(1.520143e-4f, 1.520143e-4f));
  p = __ffma2_rn(p, z, make_float2(0.0092705272f, 0.0092705272f));
  p = __ffma2_rn(p, z, make_float2(0.0422820123f, 0.0422820123f));
  p = __ffma2_rn(p, z, make_float2(0.0705230784f, 0.0705230784f));
  p = __ffma2_rn(p, z, make_float2(1.0f, 1.0f));
  float2 r = make_float2(rcp_approx(p.x), rcp_approx(p.y));
  r = __fmul2_rn(r, r);
  r = __fmul2_rn(r, r);
  r = __fmul2_rn(r, r);
  r = __fmul2_rn(r, r);
  const float2 erf_abs = __ffma2_rn(r, make_float2(-1.0f, -1.0f), make_float2(1.0f, 1.0f));
  const float2 hx = __fmul2_rn(x, make_float2(0.5f, 0.5f));
  const float2 hax = __fmul2_rn(ax, make_float2(0.5f, 0.5f));
  return __ffma2_rn(hax, erf_abs, hx);
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

// Row r of a [128][64] 16-bit slab in the 128-byte-swizzled layout TMA expects (16-byte chunk c of
// row r lives at chunk c ^ (r % 8)); conflict-free for 32 consecutive rows.
template <typename TIn>
__device__ __forceinline__ void stage_slab_row(uint8_t* slab, int r, const float (&v0)[32], const float (&v1)[32]) {
  uint32_t p[32];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    p[i] = OperandType<TIn>::pack2(v0[2 * i], v0[2 * i + 1]);
    p[16 + i] = OperandType<TIn>::pack2(v1[2 * i], v1[2 * i + 1]);
  }
  uint8_t* row = slab + r * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(row + ((c ^ (r & 7)) << 4)) = make_uint4(p[4 * c], p[4 * c + 1], p[4 * c + 2], p[4 * c + 3]);
}

// Per-thread epilogue context.
struct EpiCtx {
  uint32_t taddr;  // TMEM address: this warp's lane quarter, accumulator buffer column 0
  int row;         // tile row (TMEM lane) of this thread
  int lane, quarter, ewarp, hf;
  bool leader;     // issues the TMA stores of its column half
  uint8_t* slabs;  // 4 staging slabs: [half][2]
  float* scratch;  // same memory, used by the residual-norm epilogue
  float* tab;      // rotary rows of the current q/k tile (qkv epilogue only)
  int slot;        // next slab slot of this half (alternates 0, 1 when slots == 2)
  int slots;       // staging slabs per half: 2 (double buffered) or 1
};

// Before writing a slab: the store previously issued from it must have finished reading.
__device__ __forceinline__ uint8_t* slab_acquire(EpiCtx& e) {
  if (e.leader) {
    if (e.slots == 2)
      bulk_wait_read<1>();
    else
      bulk_wait_read<0>();
  }
  named_bar(1 + e.hf, 128);
  return e.slabs + (e.hf * e.slots + e.slot) * kSlabBytes;
}
// After writing: make the slab visible to the async proxy, then the leader stores it.
__device__ __forceinline__ void slab_release(EpiCtx& e) {
  fence_async_smem();
  named_bar(1 + e.hf, 128);
  e.slot = e.slots == 2 ? e.slot ^ 1 : 0;
}

// ------------------------------------------------------------------------------------------------ epilogues
__device__ __forceinline__ bool qkv_token(const GemmArgs& a, const TileCoord& tc, int r, int* token) {
  if (a.a_mode == A_TIME_SEQ) {
    const int t = tc.m0 + r;
    *token = (tc.b * a.T + t) * a.F + tc.f;
    return t < a.T;
  }
  const int bt = tc.m0 + (r >> 6);
  const int f = r & 63;
  *token = bt * a.F + f;
  return f < a.F && bt < a.M;
}

// Rotate 32 values (16 interleaved pairs (2j, 2j+1)) by the angles in cs[0..15], sn[0..15] (shared
// memory, 16-byte aligned): x0 c - x1 s, x1 c + x0 s.
// cs, sn: the thread's table rows (32 floats each, 16-byte chunks XOR-swizzled by swz = row & 7);
// j0 = first chunk (0 for pairs 0..15, 4 for pairs 16..31).
__device__ __forceinline__ void rotate32(float (&v)[32], const float* cs, const float* sn, int swz, int j0) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const float4 c4 = reinterpret_cast<const float4*>(cs)[(j0 + q) ^ swz];
    const float4 s4 = reinterpret_cast<const float4*>(sn)[(j0 + q) ^ swz];
    const float cc[4] = {c4.x, c4.y, c4.z, c4.w};
    const float ss[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = q * 4 + e;
      const float x0 = v[2 * j], x1 = v[2 * j + 1];
      v[2 * j] = x0 * cc[e] - x1 * ss[e];
      v[2 * j + 1] = x1 * cc[e] + x0 * ss[e];
    }
  }
}

// Rotary table rows of a row block, staged in shared memory by all epilogue warps: [cos|sin][row][32
// floats], the 16-byte chunk j of row r stored at chunk j ^ (r & 7), so a warp reading chunk j of its
// 32 rows touches every bank group (no conflicts). time mode: rows = frames t0..t0+127 (one load per
// row block); freq mode: rows = bands 0..63 (the same for every block: one load per CTA).
constexpr int kTabStride = 32;
constexpr int kTabBytes = 2 * 128 * kTabStride * 4;

__device__ __forceinline__ void load_rotary_rows(const GemmArgs& a, const TileCoord& tc, float* tab, int tid) {
  const bool time = a.a_mode == A_TIME_SEQ;
  const int L = time ? a.T : a.F;
  const int rows = time ? 128 : 64;
  const int pos0 = time ? tc.m0 : 0;
  for (int k = tid; k < 2 * rows * 8; k += 32 * kEpiWarps) {
    const int table = k / (rows * 8);
    const int rem = k - table * rows * 8;
    const int row = rem >> 3, q = rem & 7;
    const int pos = min(pos0 + row, L - 1);
    const float* src = (table == 0 ? a.cos_tab : a.sin_tab) + (size_t)pos * 32 + q * 4;
    *reinterpret_cast<float4*>(tab + (table * 128 + row) * kTabStride + ((q ^ (row & 7)) * 4)) =
        __ldg(reinterpret_cast<const float4*>(src));
  }
}

template <int BN, typename TIn>
__device__ __forceinline__ void epi_qkv(const GemmArgs& a, const TileCoord& tc, EpiCtx& e, const CUtensorMap* mq,
                                        const CUtensorMap* mk, const CUtensorMap* mv) {
  const int r = e.row;
  if (tc.n0 >= 1536) {  // gate columns (16-wide MMA): half 0 holds them
    if (e.hf == 0) {
      float v[16];
      tmem_ld16(e.taddr, v);
      int token;
      if (qkv_token(a, tc, r, &token)) {
        float g[8];
#pragma unroll
        for (int h = 0; h < 8; ++h) g[h] = sigmoidf_(v[h] + a.bias2[h]);
        float4* G = reinterpret_cast<float4*>(static_cast<float*>(a.out3) + (size_t)token * 8);
        G[0] = make_float4(g[0], g[1], g[2], g[3]);
        G[1] = make_float4(g[4], g[5], g[6], g[7]);
      }
    }
    return;
  }
  const bool time = a.a_mode == A_TIME_SEQ;
  const int part = tc.n0 >> 9;  // 0 q, 1 k, 2 v
  const CUtensorMap* map = part == 0 ? mq : part == 1 ? mk : mv;
  const int trow = time ? r : (r & 63);
  const float* cs = e.tab + trow * kTabStride;
  const float* sn = cs + 128 * kTabStride;
  const int swz = trow & 7;
#pragma unroll 1
  for (int hh = 0; hh < 2; ++hh) {
    const int hc = e.hf * 2 + hh;                    // head within the tile
    const int h = ((tc.n0 & 511) >> 6) + hc;         // head index 0..7
    uint8_t* slab = slab_acquire(e);
    float v0[32], v1[32];
    tmem_ld32(e.taddr + hc * 64, v0);
    tmem_ld32(e.taddr + hc * 64 + 32, v1);
    if (part < 2) {
      rotate32(v0, cs, sn, swz, 0);
      rotate32(v1, cs, sn, swz, 4);
    }
    stage_slab_row<TIn>(slab, r, v0, v1);
    slab_release(e);
    if (e.leader) {
      if (time)
        tma_store_3d(map, slab, 0, tc.m0, (tc.b * a.F + tc.f) * 8 + h);
      else
        tma_store_4d(map, slab, 0, 0, h, tc.m0);
      bulk_commit();
    }
  }
}

// Residual add + row L2 norm. Each warp owns 32 rows x 128 columns (its half): the accumulator goes
// through a padded shared-memory transpose 32 columns at a time, so X and xn are read and written as
// coalesced 128-byte row segments with all 32 rows' loads in flight before any store. Per-lane partial
// sums of squares are combined with a 31-shuffle transpose-reduce (row `lane` ends in lane `lane`),
// then the two halves of each row meet in shared memory.
// Residual add + RMS norm (EPI_RESNORM). Each epilogue warp owns 32 rows (its TMEM lane quarter) x 128
// columns (its half) and two 4 KB shared-memory boxes of 32 x 32 fp32 (128-byte swizzle):
//   * the warp's X boxes are loaded by TMA before the accumulator is ready (resnorm_prefetch);
//   * pass 1, per 32 columns: X_new = X + acc + b (thread = row), written back in place into the box and
//     into TMEM (over the accumulator), the box stored to X by TMA and reloaded with the chunk after next;
//   * the two halves exchange their partial sums of squares through shared memory;
//   * pass 2: xn = X_new / max(||X_new||, eps) from TMEM, 16-bit, 64 columns per box, stored by TMA.
// Rows past M are zero-filled by the loads and clipped by the stores.
constexpr int kResBoxBytes = 32 * 32 * 4;

struct ResState {
  uint8_t* box;    // this warp's two boxes
  uint64_t* xbar;  // this warp's two load barriers
  int pend[2];     // parity of the load in flight per box, -1 if none
};

__device__ __forceinline__ void resnorm_load(ResState& r, const CUtensorMap* map_x, int k, int col, int row0,
                                             int parity) {
  mbar_arrive_expect_tx(&r.xbar[k], kResBoxBytes);
  tma_load_2d(r.box + k * kResBoxBytes, map_x, &r.xbar[k], col, row0);
  r.pend[k] = parity;
}

// Issue the loads of the first two X chunks of a tile (lane 0 of each epilogue warp).
__device__ __forceinline__ void resnorm_prefetch(const GemmArgs& a, const TileCoord& tc, const EpiCtx& e,
                                                 ResState& r, const CUtensorMap* map_x) {
  const int row0 = tc.m0 + e.quarter * 32;
  if (e.lane == 0 && row0 < a.M) {  // a warp whose 32 rows all lie past M moves no data
    bulk_wait_read<0>();  // the previous tile's stores from these boxes have read them
    resnorm_load(r, map_x, 0, e.hf * 128, row0, 0);
    resnorm_load(r, map_x, 1, e.hf * 128 + 32, row0, 0);
  }
}

// Wait (bounded) for loads still in flight, so no copy lands after the CTA has exited.
__device__ __forceinline__ void resnorm_drain(const EpiCtx& e, ResState& r) {
  if (e.lane != 0) return;
  const uint64_t t0 = global_ns();
  for (int k = 0; k < 2; ++k)
    if (r.pend[k] >= 0)
      while (!mbar_try_wait(&r.xbar[k], (uint32_t)r.pend[k]) && global_ns() - t0 < kWaitLimitNs) {
      }
}

template <int BN, typename TIn>
__device__ __forceinline__ bool epi_resnorm(const GemmArgs& a, const TileCoord& tc, EpiCtx& e, ResState& r,
                                            const CUtensorMap* map_x, const CUtensorMap* map_xn, float* rs_base,
                                            int local_tile, volatile int* abort_flag) {
  static_assert(BN == 256, "the residual-norm epilogue covers whole 256-wide rows");
  const int lane = e.lane;
  const int row0 = tc.m0 + e.quarter * 32;
  const int swz = lane & 7;
  const bool live = row0 < a.M;  // a warp whose rows all lie past M only joins the barriers
  float ss = 0.f;
  bool ok = true;  // a failed wait skips the work; the decision is made collectively before bar 3
#pragma unroll 1
  for (int c = 0; c < 4 && ok && live; ++c) {
    const int k = c & 1;
    const int col = e.hf * 128 + c * 32;
    if (!mbar_wait_warp(&r.xbar[k], (uint32_t)(c >> 1), a.err, kErrWaitEpilogue, abort_flag)) {
      ok = false;
      break;
    }
    if (lane == 0) r.pend[k] = -1;
    float v[32];
    tmem_ld32(e.taddr + col, v);
    uint8_t* rowp = r.box + k * kResBoxBytes + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float4 x4 = *reinterpret_cast<const float4*>(rowp + ((j ^ swz) << 4));
      float4 b4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (a.bias) b4 = __ldg(reinterpret_cast<const float4*>(a.bias + col) + j);
      v[4 * j] += x4.x + b4.x;
      v[4 * j + 1] += x4.y + b4.y;
      v[4 * j + 2] += x4.z + b4.z;
      v[4 * j + 3] += x4.w + b4.w;
    }
#pragma unroll
    for (int i = 0; i < 32; ++i) ss = fmaf(v[i], v[i], ss);
    tmem_st32(e.taddr + col, v);  // X_new over the accumulator, read back by pass 2
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float4*>(rowp + ((j ^ swz) << 4)) =
          make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
    fence_async_smem();
    __syncwarp();
    if (lane == 0) {
      tma_store_2d(map_x, r.box + k * kResBoxBytes, col, row0);
      bulk_commit();
      if (c + 2 < 4) {
        bulk_wait_read<0>();  // the store has read the box: reuse it for the chunk after next
        resnorm_load(r, map_x, k, col + 64, row0, 1);
      }
    }
  }
  tmem_wait_st();
  // the two column halves of a row exchange their sums of squares (double buffered across tiles)
  float* rs = rs_base + (local_tile & 1) * 256;
  rs[e.hf * 128 + e.quarter * 32 + lane] = ss;
  if (!named_bar_and(3, 32 * kEpiWarps, ok)) return false;
  const float tot = rs[e.quarter * 32 + lane] + rs[128 + e.quarter * 32 + lane];
  const float inv = 1.0f / fmaxf(sqrtf(tot), a.eps);
  if (!live) return true;
  if (lane == 0) bulk_wait_read<0>();  // both boxes free for the 16-bit output
  __syncwarp();
#pragma unroll 1
  for (int k = 0; k < 2; ++k) {
    uint8_t* rowp = r.box + k * kResBoxBytes + lane * 128;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float v[32];
      tmem_ld32(e.taddr + e.hf * 128 + (2 * k + h) * 32, v);
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
      tma_store_2d(map_xn, r.box + k * kResBoxBytes, e.hf * 128 + k * 64, row0);
      bulk_commit();
    }
  }
  return true;
}

// GELU (dense) or tanh (grouped mask layer 1) on acc + bias, stored as 16-bit through TMA.
template <int BN, typename TIn>
__device__ __forceinline__ void epi_act(const GemmArgs& a, const TileCoord& tc, EpiCtx& e, const CUtensorMap* mo,
                                        bool tanh_act) {
  const float* bias = a.bias + tc.b_row;
#pragma unroll 1
  for (int hh = 0; hh < 2; ++hh) {
    const int col = e.hf * (BN / 2) + hh * 64;
    uint8_t* slab = slab_acquire(e);
    float v0[32], v1[32];
    tmem_ld32(e.taddr + col, v0);
    tmem_ld32(e.taddr + col + 32, v1);
    const float4* bp = reinterpret_cast<const float4*>(bias + col);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b0 = bp[q], b1 = bp[8 + q];
      v0[4 * q] += b0.x; v0[4 * q + 1] += b0.y; v0[4 * q + 2] += b0.z; v0[4 * q + 3] += b0.w;
      v1[4 * q] += b1.x; v1[4 * q + 1] += b1.y; v1[4 * q + 2] += b1.z; v1[4 * q + 3] += b1.w;
    }
    if (tanh_act) {
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        v0[i] = tanh_exp(v0[i]);
        v1[i] = tanh_exp(v1[i]);
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; i += 2) {
        const float2 g0 = gelu_erf2(make_float2(v0[i], v0[i + 1]));
        const float2 g1 = gelu_erf2(make_float2(v1[i], v1[i + 1]));
        v0[i] = g0.x; v0[i + 1] = g0.y;
        v1[i] = g1.x; v1[i + 1] = g1.y;
      }
    }
    stage_slab_row<TIn>(slab, e.row, v0, v1);
    slab_release(e);
    if (e.leader) {
      if (a.n_groups > 0)
        tma_store_3d(mo, slab, tc.n0 + col, tc.m0, tc.group);
      else
        tma_store_2d(mo, slab, tc.n0 + col, tc.m0);
      bulk_commit();
    }
  }
}

template <int BN>
__device__ __forceinline__ void epi_glu(const GemmArgs& a, const TileCoord& tc, EpiCtx& e) {
  const int g = tc.group;
  const int din = a.g_ncols[g] >> 1;
  const int m = tc.m0 + e.row;
  const bool valid = m < a.M;
  float* out = static_cast<float*>(a.out0) + (size_t)m * a.ld_out + a.g_outoff[g];
  const float* bias = a.bias + tc.b_row;
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    const int col = e.hf * (BN / 2) + c * 32;
    if (col >= tc.n_mma) break;  // uniform over the warp
    float v[32];
    tmem_ld32(e.taddr + col, v);
    if (valid) {
      const int col0 = tc.n0 + col;  // interleaved column: (a, g) pairs
      float r[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float av = v[2 * i] + bias[col + 2 * i];
        const float gv = v[2 * i + 1] + bias[col + 2 * i + 1];
        r[i] = av * sigmoidf_(gv);
      }
      const int c0 = col0 >> 1;  // a multiple of 16: 16-byte aligned in the row (the row stride is too)
      if (c0 + 16 <= din) {
        float4* o4 = reinterpret_cast<float4*>(out + c0);
#pragma unroll
        for (int q = 0; q < 4; ++q) o4[q] = make_float4(r[4 * q], r[4 * q + 1], r[4 * q + 2], r[4 * q + 3]);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (c0 + i < din) out[c0 + i] = r[i];
      }
    }
  }
}

// Band split + first norm (EPI_BAND): each epilogue warp owns 32 rows (frames) x 128 columns (its half)
// of one band's 256 outputs and two 4 KB shared-memory boxes (128-byte swizzle), stored by TMA into the
// 3-D views X (256, bands, rows) fp32 and xn (256, bands, rows) 16-bit, so every global write is a whole
// line. Pass 1: X = acc + b, 32 columns per box, and the row's sum of squares; the two column halves meet
// in shared memory; pass 2: xn = X / max(|X|, eps) from a second read of the accumulator, 64 columns
// per box. Returns false if the row-sum exchange was abandoned (a failed wait elsewhere).
template <int BN, typename TIn>
__device__ __forceinline__ bool epi_band(const GemmArgs& a, const TileCoord& tc, EpiCtx& e, uint8_t* box,
                                         const CUtensorMap* map_x, const CUtensorMap* map_xn, float* rs_base,
                                         int local_tile) {
  static_assert(BN == 256, "the band epilogue covers whole 256-wide rows");
  const int lane = e.lane;
  const int row0 = tc.m0 + e.quarter * 32;
  const bool live = row0 < a.M;  // a warp whose 32 rows all lie past M stores nothing
  const int swz = lane & 7;
  const float* bias = a.bias + tc.group * 256 + e.hf * 128;
  if (lane == 0) bulk_wait_read<0>();  // the previous tile's stores have read both boxes
  __syncwarp();
  float ss = 0.f;
#pragma unroll 1
  for (int c = 0; c < 4; ++c) {
    uint8_t* rowp = box + (c & 1) * kResBoxBytes + lane * 128;
    if (c >= 2) {  // the store from this box two chunks ago has read it
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
    }
    float v[32];
    tmem_ld32(e.taddr + e.hf * 128 + c * 32, v);
    const float4* b4 = reinterpret_cast<const float4*>(bias + c * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = __ldg(b4 + q);
      const float4 x = make_float4(v[4 * q] + b.x, v[4 * q + 1] + b.y, v[4 * q + 2] + b.z, v[4 * q + 3] + b.w);
      ss = fmaf(x.x, x.x, fmaf(x.y, x.y, fmaf(x.z, x.z, fmaf(x.w, x.w, ss))));
      *reinterpret_cast<float4*>(rowp + ((q ^ swz) << 4)) = x;
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0 && live) {
      tma_store_3d(map_x, box + (c & 1) * kResBoxBytes, e.hf * 128 + c * 32, tc.group, row0);
      bulk_commit();
    }
  }
  float* rs = rs_base + (local_tile & 1) * 256;
  rs[e.hf * 128 + e.quarter * 32 + lane] = ss;
  if (!named_bar_and(3, 32 * kEpiWarps, true)) return false;
  const float tot = rs[e.quarter * 32 + lane] + rs[128 + e.quarter * 32 + lane];
  const float inv = 1.0f / fmaxf(sqrtf(tot), a.eps);
  if (lane == 0) bulk_wait_read<0>();  // both boxes free for the 16-bit output
  __syncwarp();
#pragma unroll 1
  for (int k = 0; k < 2; ++k) {
    uint8_t* rowp = box + k * kResBoxBytes + lane * 128;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float v[32];
      tmem_ld32(e.taddr + e.hf * 128 + (2 * k + h) * 32, v);
      const float4* b4 = reinterpret_cast<const float4*>(bias + (2 * k + h) * 32);
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float4 b0 = __ldg(b4 + 2 * t), b1 = __ldg(b4 + 2 * t + 1);
        uint4 u;
        u.x = OperandType<TIn>::pack2((v[8 * t] + b0.x) * inv, (v[8 * t + 1] + b0.y) * inv);
        u.y = OperandType<TIn>::pack2((v[8 * t + 2] + b0.z) * inv, (v[8 * t + 3] + b0.w) * inv);
        u.z = OperandType<TIn>::pack2((v[8 * t + 4] + b1.x) * inv, (v[8 * t + 5] + b1.y) * inv);
        u.w = OperandType<TIn>::pack2((v[8 * t + 6] + b1.z) * inv, (v[8 * t + 7] + b1.w) * inv);
        *reinterpret_cast<uint4*>(rowp + (((h * 4 + t) ^ swz) << 4)) = u;
      }
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0 && live) {
      tma_store_3d(map_xn, box + k * kResBoxBytes, e.hf * 128 + k * 64, tc.group, row0);
      bulk_commit();
    }
  }
  return true;
}

// Plain fp32 output (EPI_F32): Y = acc + b. Each epilogue warp owns 32 rows x its half of the columns and
// two 4 KB boxes (32 x 32 fp32, 128-byte swizzle), stored by TMA into Y, 2-D (N, rows) or for grouped
// GEMMs 3-D (N, groups, rows); chunks at or past the tile's valid width are skipped.
template <int BN>
__device__ __forceinline__ void epi_f32(const GemmArgs& a, const TileCoord& tc, EpiCtx& e, uint8_t* box,
                                        const CUtensorMap* map_y) {
  const int lane = e.lane;
  const int row0 = tc.m0 + e.quarter * 32;
  const bool live = row0 < a.M;
  const int swz = lane & 7;
  const float* bias = a.bias ? a.bias + (size_t)tc.group * a.bias_gstride + tc.n0 : nullptr;
  if (lane == 0) bulk_wait_read<0>();  // the previous tile's stores have read both boxes
  __syncwarp();
#pragma unroll 1
  for (int c = 0; c < BN / 64; ++c) {
    const int col = e.hf * (BN / 2) + c * 32;
    if (col >= tc.n_valid) break;  // uniform over the warp
    uint8_t* rowp = box + (c & 1) * kResBoxBytes + lane * 128;
    if (c >= 2) {  // the store from this box two chunks ago has read it
      if (lane == 0) bulk_wait_read<1>();
      __syncwarp();
    }
    float v[32];
    tmem_ld32(e.taddr + col, v);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 b = bias ? __ldg(reinterpret_cast<const float4*>(bias + col) + q) : make_float4(0.f, 0.f, 0.f, 0.f);
      *reinterpret_cast<float4*>(rowp + ((q ^ swz) << 4)) =
          make_float4(v[4 * q] + b.x, v[4 * q + 1] + b.y, v[4 * q + 2] + b.z, v[4 * q + 3] + b.w);
    }
    fence_async_smem();
    __syncwarp();
    if (lane == 0 && live) {
      if (a.n_groups > 0)
        tma_store_3d(map_y, box + (c & 1) * kResBoxBytes, tc.n0 + col, tc.group, row0);
      else
        tma_store_2d(map_y, box + (c & 1) * kResBoxBytes, tc.n0 + col, row0);
      bulk_commit();
    }
  }
}

// ------------------------------------------------------------------------------------------------ kernel
template <int BN, int STAGES, int EPI>
struct GemmSmem {
  // qkv keeps its A tile (K = 256) resident while it makes all N tiles of a row block, so only B streams
  static constexpr bool kAStat = EPI == EPI_QKV;
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int kBBytes = BN * kGemmBK * 2;       // 32 KB at BN = 256
  static constexpr int kAResBytes = kAStat ? 4 * kABytes : 0;
  static constexpr int kStageBytes = kAStat ? kBBytes : kABytes + kBBytes;
  static constexpr int kStageOffset = kAResBytes;
  static constexpr int kOutOffset = kStageOffset + STAGES * kStageBytes;  // staging slabs / residual-norm boxes
  static constexpr int kSlabsPerHalf = 2;  // double-buffered staging slabs per column half
  static constexpr int kOutBytes = 2 * kSlabsPerHalf * kSlabBytes;
  static_assert(EPI != EPI_RESNORM || kEpiWarps * 2 * kResBoxBytes <= kOutBytes, "residual-norm boxes must fit");
  static constexpr int kTabOffset = kOutOffset + kOutBytes;  // rotary rows (qkv only)
  static constexpr int kRsOffset = kTabOffset + (is_qkv(EPI) ? kTabBytes : 0);  // row sums (norm epilogues)
  static constexpr int kBarOffset = kRsOffset + (EPI == EPI_RESNORM || EPI == EPI_BAND ? 2 * 256 * 4 : 0);
  static constexpr int kBytes = kBarOffset + 256 + 1024;  // + barriers + alignment slack
  static_assert(kBytes <= 232448, "shared memory per CTA");
};

template <int BN, int STAGES, int EPI, typename TIn>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                const __grid_constant__ CUtensorMap map_o0, const __grid_constant__ CUtensorMap map_o1,
                const __grid_constant__ CUtensorMap map_o2, const __grid_constant__ GemmArgs args) {
  using S = GemmSmem<BN, STAGES, EPI>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::kBarOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* xbars = drain + 2;  // residual-norm X loads: [epilogue warp][2]
  uint64_t* a_full = drain + 2;   // qkv: resident A tile loaded (same slots as xbars, another kernel)
  uint64_t* a_empty = drain + 3;  // qkv: the MMAs of the row block have read the A tile
  // qkv walks row blocks (groups of n_tiles consecutive tiles); other epilogues walk single tiles
  const int n_units = S::kAStat ? args.num_tiles / args.n_tiles : args.num_tiles;
  const int tiles_per_unit = S::kAStat ? args.n_tiles : 1;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int a_dims = (args.a_mode == A_ROWS || args.a_mode == A_BAND) ? 2 : args.a_mode == A_TIME_SEQ ? 4 : 3;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 32 * kEpiWarps);
    }
    mbar_init(drain, 1);
    if constexpr (EPI == EPI_RESNORM)
      for (int b = 0; b < 2 * kEpiWarps; ++b) mbar_init(&xbars[b], 1);
    if constexpr (S::kAStat) {
      mbar_init(a_full, 1);
      mbar_init(a_empty, 1);
    }
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
      int lu = 0;       // units of this CTA so far (qkv: row blocks, a_full / a_empty phases)
      int a_loads = 0;  // qkv: resident A tiles requested
      for (int unit = blockIdx.x; unit < n_units && ok; unit += gridDim.x, ++lu) {
        if constexpr (S::kAStat) {
          // the resident A tile of this row block (all k blocks), once the previous block's MMAs read theirs
          const TileCoord t0 = gemm_decode<BN>(args, unit * tiles_per_unit);
          if (!mbar_wait(a_empty, ((uint32_t)lu & 1) ^ 1, args.err, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(a_full, args.k_blocks * S::kABytes);
          ++a_loads;
          for (int kb = 0; kb < args.k_blocks; ++kb) {
            uint8_t* sa = smem + kb * S::kABytes;
            const int kx = kb * kGemmBK;
            if (a_dims == 2)
              tma_load_2d(sa, &map_a, a_full, kx, t0.a1);
            else if (a_dims == 3)
              tma_load_3d(sa, &map_a, a_full, kx, t0.a1, t0.a2);
            else
              tma_load_4d(sa, &map_a, a_full, kx, t0.a1, t0.a2, t0.a3);
          }
        }
        for (int u = 0; u < tiles_per_unit && ok; ++u) {
        const TileCoord tc = gemm_decode<BN>(args, unit * tiles_per_unit + u);
        for (int kb = 0; kb < tc.kblocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, args.err, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + S::kStageOffset + stage * S::kStageBytes;
          mbar_arrive_expect_tx(&full[stage], S::kStageBytes);
          const int kx = tc.koff + kb * kGemmBK;
          if constexpr (S::kAStat) {
            tma_load_2d(st, &map_b, &full[stage], kx, tc.b_row);
          } else {
            uint8_t* sb = st + S::kABytes;
            if (a_dims == 2)
              tma_load_2d(st, &map_a, &full[stage], kx, tc.a1);
            else if (a_dims == 3)
              tma_load_3d(st, &map_a, &full[stage], kx, tc.a1, tc.a2);
            else
              tma_load_4d(st, &map_a, &full[stage], kx, tc.a1, tc.a2, tc.a3);
            tma_load_2d(sb, &map_b, &full[stage], kx, tc.b_row);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        }
      }
      if (!ok) {  // drain the copies still in flight before the CTA's shared memory is released
        for (int j = max(0, issued - STAGES); j < issued; ++j) {
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1) && global_ns() - t0 < kWaitLimitNs) {
          }
        }
        if (a_loads > 0) {
          const uint64_t t0 = global_ns();
          while (!mbar_try_wait(a_full, (uint32_t)(a_loads - 1) & 1) && global_ns() - t0 < kWaitLimitNs) {
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0, lu = 0;
      bool ok = true;
      const uint32_t a_res = smem_u32(smem);  // qkv: resident A tile
      for (int unit = blockIdx.x; unit < n_units && ok; unit += gridDim.x, ++lu) {
        if constexpr (S::kAStat) {
          if (!mbar_wait(a_full, (uint32_t)lu & 1, args.err, kErrWaitMma, abort_flag)) {
            ok = false;
            break;
          }
        }
        for (int u = 0; u < tiles_per_unit && ok; ++u, ++local) {
        const TileCoord tc = gemm_decode<BN>(args, unit * tiles_per_unit + u);
        const int buf = local & 1;
        const uint32_t use = (uint32_t)(local >> 1);
        if (!mbar_wait(&acc_empty[buf], (use & 1) ^ 1, args.err, kErrWaitMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(buf * BN);
        const uint32_t idesc = idesc_f16(kGemmBM, tc.n_mma, OperandType<TIn>::kFormat, 0, 0);
        for (int kb = 0; kb < tc.kblocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, args.err, kErrWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t st = smem_u32(smem + S::kStageOffset + stage * S::kStageBytes);
          const uint32_t sa = S::kAStat ? a_res + kb * S::kABytes : st;
          const uint32_t sb = S::kAStat ? st : st + S::kABytes;
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
        if constexpr (S::kAStat) mma_commit(a_empty);  // this row block's MMAs have read the A tile
      }
      // all MMAs issued by this thread are complete once `drain` fires
      mma_commit(drain);
      const uint64_t t0 = global_ns();
      while (!mbar_try_wait(drain, 0) && global_ns() - t0 < kWaitLimitNs) {
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2-9)
    EpiCtx e;
    e.lane = lane;
    e.quarter = warp & 3;
    e.ewarp = warp - 2;
    e.hf = e.ewarp >> 2;
    e.row = e.quarter * 32 + lane;
    e.leader = (e.ewarp & 3) == 0 && lane == 0;
    e.slabs = smem + S::kOutOffset;
    e.scratch = reinterpret_cast<float*>(smem + S::kOutOffset);
    e.tab = reinterpret_cast<float*>(smem + S::kTabOffset);
    e.slot = 0;
    e.slots = S::kSlabsPerHalf;
    ResState rst;
    rst.box = smem + S::kOutOffset + e.ewarp * 2 * kResBoxBytes;
    rst.xbar = xbars + e.ewarp * 2;
    rst.pend[0] = rst.pend[1] = -1;
    int local = 0;
    bool run = true;
    for (int unit = blockIdx.x; unit < n_units && run; unit += gridDim.x) {
    for (int u = 0; u < tiles_per_unit; ++u, ++local) {
      const TileCoord tc = gemm_decode<BN>(args, unit * tiles_per_unit + u);
      const int buf = local & 1;
      const uint32_t use = (uint32_t)(local >> 1);
      if constexpr (EPI == EPI_RESNORM) resnorm_prefetch(args, tc, e, rst, &map_o0);  // overlaps this tile's MMAs
      if constexpr (is_qkv(EPI)) {
        // the row block's rotary rows, staged while its first tile's MMAs run: time mode once per row
        // block (frames m0..m0+127), freq mode once per CTA (bands 0..63 for every block)
        if (u == 0 && (args.a_mode == A_TIME_SEQ || local == 0)) {
          named_bar(3, 32 * kEpiWarps);  // every warp is done with the previous table
          load_rotary_rows(args, tc, e.tab, e.ewarp * 32 + lane);
          named_bar(3, 32 * kEpiWarps);
        }
      }
      // every epilogue warp takes the same decision, so no warp is left waiting at a named barrier
      const bool ok = mbar_wait_warp(&acc_full[buf], use & 1, args.err, kErrWaitEpilogue, abort_flag);
      if (!named_bar_and(4, 32 * kEpiWarps, ok)) {
        run = false;
        break;
      }
      tc_fence_after();
      e.taddr = tmem_base + (uint32_t)(buf * BN) + ((uint32_t)(e.quarter * 32) << 16);
      if constexpr (is_qkv(EPI)) {
        epi_qkv<BN, TIn>(args, tc, e, &map_o0, &map_o1, &map_o2);
      } else if constexpr (EPI == EPI_RESNORM) {
        const bool ok2 = epi_resnorm<BN, TIn>(args, tc, e, rst, &map_o0, &map_o1,
                                              reinterpret_cast<float*>(smem + S::kRsOffset), local, abort_flag);
        if (!named_bar_and(4, 32 * kEpiWarps, ok2)) {
          run = false;
          break;
        }
      } else if constexpr (EPI == EPI_GELU) {
        epi_act<BN, TIn>(args, tc, e, &map_o0, false);
      } else if constexpr (EPI == EPI_MASK_TANH) {
        epi_act<BN, TIn>(args, tc, e, &map_o0, true);
      } else if constexpr (EPI == EPI_F32) {
        epi_f32<BN>(args, tc, e, rst.box, &map_o0);
      } else if constexpr (EPI == EPI_BAND) {
        if (!epi_band<BN, TIn>(args, tc, e, rst.box, &map_o0, &map_o1, reinterpret_cast<float*>(smem + S::kRsOffset),
                               local)) {
          run = false;
          break;
        }
      } else {
        epi_glu<BN>(args, tc, e);
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[buf]);
    }
    }
    if constexpr (EPI == EPI_RESNORM || EPI == EPI_BAND || EPI == EPI_F32) {
      if constexpr (EPI == EPI_RESNORM) resnorm_drain(e, rst);
      if (lane == 0) bulk_wait<0>();  // this warp's stores have completed
    } else {
      if (e.leader) bulk_wait<0>();  // this half's output stores have completed
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
