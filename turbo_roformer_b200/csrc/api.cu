// C ABI of libtrcuda.so (declared in include/trcuda.h): model handle, load-time weight folding,
// TMA descriptors, work buffers and the forward orchestration.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/trcuda.h"
#include "attention.cuh"
#include "attention_time.cuh"
#include "gemm.cuh"
#include "internal.h"
#include "mlp.cuh"

namespace {

using trc::AttnArgs;
using trc::GemmArgs;

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

}  // namespace

namespace trc {
int set_last_error(int code, const char* msg) { return fail(code, "%s", msg); }
}  // namespace trc

namespace {

#define TRC_CUDA(call)                                                                              \
  do {                                                                                              \
    cudaError_t e_ = (call);                                                                        \
    if (e_ != cudaSuccess) return fail(TRC_E_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

// ------------------------------------------------------------------------------------------------ TMA maps
using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// Element type code of make_map beyond TRC_PREC_FP16 / TRC_PREC_BF16.
constexpr int kMapF32 = 2;

// Row-major tensor of 16-bit (precision = TRC_PREC_*) or fp32 (kMapF32) elements: dims[0] innermost
// (elements), strides in bytes for dims[1..rank-1]. 128-byte swizzle, zero fill for out-of-range rows.
int make_map(CUtensorMap* m, int precision, const void* ptr, int rank, const uint64_t* dims,
             const uint64_t* strides_bytes, const uint32_t* box) {
  EncodeFn fn = encode_fn();
  if (!fn) return fail(TRC_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (reinterpret_cast<uintptr_t>(ptr) % 16) return fail(TRC_E_INVALID, "TMA base address not 16-byte aligned");
  for (int i = 0; i < rank - 1; ++i)
    if (strides_bytes[i] % 16) return fail(TRC_E_INVALID, "TMA stride not a multiple of 16 bytes");
  cuuint64_t gd[5], gs[4];
  cuuint32_t bd[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bd[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i < rank - 1; ++i) gs[i] = strides_bytes[i];
  const CUtensorMapDataType dt = precision == kMapF32         ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                 : precision == TRC_PREC_FP16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                              : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16;
  CUresult r = fn(m, dt, (cuuint32_t)rank, const_cast<void*>(ptr), gd, gs, bd, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TRC_E_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return TRC_OK;
}

// Cached variant for the forward path (keyed on everything that defines the map).
int make_map_cached(trc_handle* h, CUtensorMap* m, const void* ptr, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int dtype = -1);

// [rows][cols] with box (64, box_rows)
int map_2d(CUtensorMap* m, int prec, const void* p, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t st[1] = {cols * 2};
  const uint32_t box[2] = {64, box_rows};
  return make_map(m, prec, p, 2, dims, st, box);
}

// ------------------------------------------------------------------------------------------------ host fp16
uint16_t to_bits(float x, int prec) {
  if (prec == TRC_PREC_FP16) {
    __half h = __float2half_rn(x);
    uint16_t u;
    std::memcpy(&u, &h, 2);
    return u;
  }
  __nv_bfloat16 h = __float2bfloat16_rn(x);
  uint16_t u;
  std::memcpy(&u, &h, 2);
  return u;
}

template <typename T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
  int alloc(size_t count) {
    if (count <= n && p) return TRC_OK;
    if (p) cudaFree(p);
    p = nullptr;
    n = 0;
    if (cudaMalloc(&p, count * sizeof(T) + 256) != cudaSuccess) {
      cudaGetLastError();
      return fail(TRC_E_NOMEM, "cudaMalloc of %zu bytes failed", count * sizeof(T));
    }
    n = count;
    return TRC_OK;
  }
  int upload(const std::vector<T>& h) {
    int rc = alloc(h.size());
    if (rc) return rc;
    TRC_CUDA(cudaMemcpy(p, h.data(), h.size() * sizeof(T), cudaMemcpyHostToDevice));
    return TRC_OK;
  }
};

struct LayerDev {
  DevBuf<uint16_t> wqkv;  // [1544][256] folded q|k|v|gates
  DevBuf<float> gbias;    // [8]
  DevBuf<uint16_t> wo;    // [256][512]
  DevBuf<uint16_t> w1;    // [ff][256] folded
  DevBuf<float> b1;       // [ff]
  DevBuf<uint16_t> w2;    // [256][ff]
  DevBuf<float> b2;       // [256]
  CUtensorMap m_wqkv, m_wo, m_w1, m_w2;
  CUtensorMap m_w1c;  // W1 in 128-row boxes (hidden chunks of the fused feed-forward kernel)
};

struct Tables {
  DevBuf<float> cos_t, sin_t;  // [L][32]
};

}  // namespace

struct trc_handle {
  // configuration
  int dim = 256, depth = 0, heads = 8, dim_head = 64, ff = 1024, nb = 0, n_fft = 0, hop = 0, hidden = 0;
  int prec = TRC_PREC_FP16;
  int device = 0;
  int num_sms = 148;
  std::vector<int> freqs;     // per band
  std::vector<int> band_off;  // prefix of 4 * freqs (nb + 1)
  std::vector<int> m2_off;    // prefix of 8 * freqs (interleaved mask layer-2 rows)
  int width = 0;              // 4 * (n_fft / 2 + 1)
  // weights
  std::map<std::string, std::vector<float>> params;
  bool prepared = false;
  std::vector<std::unique_ptr<LayerDev>> layers;
  std::vector<float> rot_freqs[2];
  std::map<std::pair<int, int>, std::unique_ptr<Tables>> tables;
  // band split as a grouped GEMM: W' [256][bs_kp] 16-bit, band k in columns [pad_off[k], pad_off[k+1])
  DevBuf<uint16_t> bs_w;
  DevBuf<float> bs_bias;         // [nb][256]
  DevBuf<int> bs_off, bs_poff;   // band_off, pad_off (nb + 1 each)
  std::vector<int> pad_off;      // prefix of the band widths rounded up to 64 columns
  int bs_kp = 0;
  CUtensorMap m_bs_w;
  DevBuf<uint16_t> mk_w1, mk_w2;
  DevBuf<float> mk_b1, mk_b2;
  CUtensorMap m_mk_w1, m_mk_w2;
  DevBuf<float> window;
  DevBuf<float2> tw_fwd, tw_inv;
  DevBuf<int> err;
  // forward work buffers (sized for ws_B x ws_T)
  int ws_B = 0, ws_T = 0;
  DevBuf<float> xin, X, mask, frames;
  DevBuf<float> Y;  // fp32 residual branch [rows][dim] (models whose width is not 256)
  DevBuf<uint16_t> bs_a;  // normalised, padded band inputs [rows][bs_kp]
  DevBuf<uint16_t> xn, Q, K, V, O, H;
  DevBuf<float> G;
  // tensor maps by (pointer, precision, rank, dims, strides, box): work buffers are stable, so most hit
  std::map<std::vector<uint64_t>, CUtensorMap> map_cache;
  // section timing (CUDA events on the launch stream, like the reference's per-section _Timer)
  bool timing = false;
  std::vector<cudaEvent_t> ev_pool;
  std::vector<std::pair<std::string, std::pair<cudaEvent_t, cudaEvent_t>>> ev_pending;
  std::map<std::string, std::pair<double, long>> section;  // name -> (ms, launches)
  ~trc_handle() {
    for (auto& e : ev_pool) cudaEventDestroy(e);
    for (auto& p : ev_pending) {
      cudaEventDestroy(p.second.first);
      cudaEventDestroy(p.second.second);
    }
  }
};

namespace {

std::atomic<long long> g_launches{0};

}  // namespace

namespace trc {
void count_launches(int n) { g_launches += n; }
}  // namespace trc

namespace {

cudaEvent_t pool_event(trc_handle* h) {
  if (!h->ev_pool.empty()) {
    cudaEvent_t e = h->ev_pool.back();
    h->ev_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  cudaEventCreate(&e);
  return e;
}

// Times one stage on `st` when the handle's timing is on; counts the kernel launches it makes.
struct Section {
  trc_handle* h;
  const char* name;
  cudaStream_t st;
  int launches;
  cudaEvent_t e0 = nullptr;
  Section(trc_handle* h_, const char* n, cudaStream_t s_, int l = 1) : h(h_), name(n), st(s_), launches(l) {
    if (h->timing) {
      e0 = pool_event(h);
      cudaEventRecord(e0, st);
    }
  }
  ~Section() {
    g_launches += launches;
    if (h->timing && e0) {
      cudaEvent_t e1 = pool_event(h);
      cudaEventRecord(e1, st);
      h->ev_pending.push_back({name, {e0, e1}});
      h->section[name].second += launches;
      if (h->ev_pending.size() >= 512) harvest(h);
    }
  }
  // Fold finished event pairs (oldest first, non-blocking) into the totals and recycle the events, so
  // long timed runs never create events on the launch path.
  static void harvest(trc_handle* h) {
    size_t k = 0;
    for (; k < h->ev_pending.size(); ++k) {
      auto& p = h->ev_pending[k];
      if (cudaEventQuery(p.second.second) != cudaSuccess) break;
      float ms = 0.f;
      if (cudaEventElapsedTime(&ms, p.second.first, p.second.second) == cudaSuccess) h->section[p.first].first += ms;
      h->ev_pool.push_back(p.second.first);
      h->ev_pool.push_back(p.second.second);
    }
    cudaGetLastError();  // a not-ready query leaves cudaErrorNotReady behind
    h->ev_pending.erase(h->ev_pending.begin(), h->ev_pending.begin() + k);
  }
};

int make_map_cached(trc_handle* h, CUtensorMap* m, const void* ptr, int rank, const uint64_t* dims,
                    const uint64_t* strides_bytes, const uint32_t* box, int dtype) {
  if (dtype < 0) dtype = h->prec;
  std::vector<uint64_t> key;
  key.reserve(16);
  key.push_back(reinterpret_cast<uint64_t>(ptr));
  key.push_back((uint64_t)dtype);
  key.push_back((uint64_t)rank);
  for (int i = 0; i < rank; ++i) key.push_back(dims[i]);
  for (int i = 0; i < rank - 1; ++i) key.push_back(strides_bytes[i]);
  for (int i = 0; i < rank; ++i) key.push_back(box[i]);
  auto it = h->map_cache.find(key);
  if (it != h->map_cache.end()) {
    *m = it->second;
    return TRC_OK;
  }
  const int rc = make_map(m, dtype, ptr, rank, dims, strides_bytes, box);
  if (rc == TRC_OK) {
    if (h->map_cache.size() > 4096) h->map_cache.clear();
    h->map_cache[key] = *m;
  }
  return rc;
}

int map_2d_cached(trc_handle* h, CUtensorMap* m, const void* p, uint64_t cols, uint64_t rows, uint32_t box_rows) {
  const uint64_t dims[2] = {cols, rows};
  const uint64_t st[1] = {cols * 2};
  const uint32_t box[2] = {64, box_rows};
  return make_map_cached(h, m, p, 2, dims, st, box);
}

const std::vector<float>* param(trc_handle* h, const std::string& name, size_t numel) {
  auto it = h->params.find(name);
  if (it == h->params.end()) {
    fail(TRC_E_INVALID, "missing parameter %s", name.c_str());
    return nullptr;
  }
  if (it->second.size() != numel) {
    fail(TRC_E_INVALID, "parameter %s has %zu elements, expected %zu", name.c_str(), it->second.size(), numel);
    return nullptr;
  }
  return &it->second;
}

int upload_bits(DevBuf<uint16_t>& d, const std::vector<float>& v, int prec) {
  std::vector<uint16_t> b(v.size());
  for (size_t i = 0; i < v.size(); ++i) b[i] = to_bits(v[i], prec);
  return d.upload(b);
}

// Rotary cos/sin tables [L][32] for a mode: angle = float(pos) * freq in fp32 like the reference
// (fast.py:193-199), cos/sin evaluated in double and rounded once.
Tables* get_tables(trc_handle* h, int mode, int L) {
  auto key = std::make_pair(mode, L);
  auto it = h->tables.find(key);
  if (it != h->tables.end()) return it->second.get();
  auto t = std::make_unique<Tables>();
  std::vector<float> c((size_t)L * 32), s((size_t)L * 32);
  for (int p = 0; p < L; ++p)
    for (int i = 0; i < 32; ++i) {
      const float ang = (float)p * h->rot_freqs[mode][i];
      c[(size_t)p * 32 + i] = (float)std::cos((double)ang);
      s[(size_t)p * 32 + i] = (float)std::sin((double)ang);
    }
  if (t->cos_t.upload(c) || t->sin_t.upload(s)) return nullptr;
  Tables* raw = t.get();
  h->tables[key] = std::move(t);
  return raw;
}

int ensure_workspace(trc_handle* h, int B, int T) {
  if (B <= h->ws_B && T <= h->ws_T) return TRC_OK;
  const int nB = B > h->ws_B ? B : h->ws_B;
  const int nT = T > h->ws_T ? T : h->ws_T;
  const size_t BT = (size_t)nB * nT;
  const size_t N = BT * h->nb;
  const size_t hid = (size_t)(h->ff > h->hidden ? h->ff : h->hidden);
  int rc;
  if ((rc = h->xin.alloc(BT * h->width)) || (rc = h->mask.alloc(BT * h->width)) ||
      (rc = h->frames.alloc(BT * 2 * h->n_fft)) || (rc = h->X.alloc(N * h->dim)) || (rc = h->xn.alloc(N * h->dim)) ||
      (h->dim != 256 && (rc = h->Y.alloc(N * h->dim))) ||
      (rc = h->Q.alloc(N * 512)) || (rc = h->K.alloc(N * 512)) || (rc = h->V.alloc(N * 512)) ||
      (rc = h->O.alloc(N * 512)) || (rc = h->H.alloc(N * hid)) || (rc = h->G.alloc(N * 8)) ||
      (rc = h->bs_a.alloc(BT * h->bs_kp)))
    return rc;
  h->ws_B = nB;
  h->ws_T = nT;
  return TRC_OK;
}

int check_launch(cudaError_t e, const char* what) {
  if (e != cudaSuccess) return fail(TRC_E_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
  return TRC_OK;
}

GemmArgs dense_args(trc_handle* h, int64_t rows, int n_cols, int k) {
  GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  const int m_tiles = (int)((rows + 127) / 128);
  a.n_tiles = (n_cols + 255) / 256;
  a.num_tiles = m_tiles * a.n_tiles;
  a.k_blocks = k / 64;
  a.a_mode = trc::A_ROWS;
  a.M = (int)rows;
  a.N = n_cols;
  a.n_groups = 0;
  a.eps = 1e-12f;
  a.err = h->err.p;
  return a;
}

// Q/K/V tensor maps of the attention layout. time: 3-D (64, T, B*F*8), box (64, 128, 1) = 128 frames of
// one (batch, band, head) sequence; freq: 4-D (64, F, 8, B*T), box (64, 64, 1, 2) = two frames' band
// sequences of one head (rows f >= F are clipped / zero-filled).
int qkv_map(trc_handle* h, CUtensorMap* m, const void* p, int mode, int B, int T) {
  const int F = h->nb;
  if (mode == 0) {
    const uint64_t dims[3] = {64, (uint64_t)T, (uint64_t)B * F * 8};
    const uint64_t st[2] = {128, (uint64_t)T * 128};
    const uint32_t box[3] = {64, 128, 1};
    return make_map_cached(h, m, p, 3, dims, st, box);
  }
  const uint64_t dims[4] = {64, (uint64_t)F, 8, (uint64_t)B * T};
  const uint64_t st[3] = {128, (uint64_t)F * 128, (uint64_t)F * 8 * 128};
  const uint32_t box[4] = {64, 64, 1, 2};
  return make_map_cached(h, m, p, 4, dims, st, box);
}

int run_qkv(trc_handle* h, int layer, const void* xn, int B, int T, void* Q, void* K, void* V, float* G,
            cudaStream_t st) {
  const int mode = layer & 1;
  const int F = h->nb;
  const int L = mode == 0 ? T : F;
  if (F > 64) return fail(TRC_E_INVALID, "at most 64 bands are supported");
  Tables* tab = get_tables(h, mode, L);
  if (!tab) return TRC_E_CUDA;
  LayerDev& lw = *h->layers[layer];
  CUtensorMap ma, mo[3];
  int rc;
  const int D = h->dim;
  GemmArgs a = dense_args(h, 1, 1544, D);
  if (mode == 0) {  // A rows: 128 consecutive frames of one band, xn viewed as (k, band, frame, batch)
    const uint64_t dims[4] = {(uint64_t)D, (uint64_t)F, (uint64_t)T, (uint64_t)B};
    const uint64_t strides[3] = {(uint64_t)D * 2, (uint64_t)F * D * 2, (uint64_t)T * F * D * 2};
    const uint32_t box[4] = {64, 1, 128, 1};
    if ((rc = make_map_cached(h, &ma, xn, 4, dims, strides, box))) return rc;
    a.a_mode = trc::A_TIME_SEQ;
    a.M = T;
    a.m_tiles = (T + 127) / 128;
    a.num_tiles = B * F * a.m_tiles * a.n_tiles;
  } else {  // A rows: two frames x 64 band slots, xn viewed as (k, band, frame)
    const uint64_t dims[3] = {(uint64_t)D, (uint64_t)F, (uint64_t)B * T};
    const uint64_t strides[2] = {(uint64_t)D * 2, (uint64_t)F * D * 2};
    const uint32_t box[3] = {64, 64, 2};
    if ((rc = make_map_cached(h, &ma, xn, 3, dims, strides, box))) return rc;
    a.a_mode = trc::A_FREQ_PAIR;
    a.M = B * T;
    a.num_tiles = ((B * T + 1) / 2) * a.n_tiles;
  }
  if ((rc = qkv_map(h, &mo[0], Q, mode, B, T)) || (rc = qkv_map(h, &mo[1], K, mode, B, T)) ||
      (rc = qkv_map(h, &mo[2], V, mode, B, T)))
    return rc;
  a.out0 = Q;
  a.out1 = K;
  a.out2 = V;
  a.out3 = G;
  a.bias2 = lw.gbias.p;
  a.cos_tab = tab->cos_t.p;
  a.sin_tab = tab->sin_t.p;
  a.T = T;
  a.F = F;
  // a 256-wide row block stays resident in shared memory for all 7 column tiles; wider ones stream with B
  return check_launch(trc::launch_gemm(D == 256 ? trc::EPI_QKV : trc::EPI_QKVS, h->prec, ma, lw.m_wqkv, mo, a,
                                       h->num_sms, st),
                      "qkv gemm");
}

int run_attention(trc_handle* h, int mode, const void* Q, const void* K, const void* V, const float* G, void* O,
                  int B, int T, cudaStream_t st) {
  const int F = h->nb;
  AttnArgs a;
  std::memset(&a, 0, sizeof(a));
  a.mode = mode;
  a.T = T;
  a.F = F;
  a.G = G;
  a.O = O;
  a.err = h->err.p;
  uint64_t dims[3], strides[2];
  uint32_t box[3];
  if (mode == 0) {
    a.L = T;
    a.BH = B * F * 8;
    const int q_tiles = (T + 127) / 128;
    a.q_pairs = (q_tiles + trc::kTaTiles - 1) / trc::kTaTiles;  // items of three query tiles
    a.n_kv = (T + 63) / 64;                                        // 64-key steps
    a.num_items = a.BH * a.q_pairs;
    box[0] = 64; box[1] = 128; box[2] = 1;
  } else {
    if (F > 64) return fail(TRC_E_INVALID, "freq attention supports at most 64 bands");
    a.L = F;
    a.BH = B * T * 8;
    a.q_pairs = 1;
    a.n_kv = 1;
    a.num_items = (a.BH + 3) / 4;
    box[0] = 64; box[1] = 64; box[2] = 2;
  }
  dims[0] = 64;
  dims[1] = (uint64_t)a.L;
  dims[2] = (uint64_t)a.BH;
  strides[0] = 128;
  strides[1] = (uint64_t)a.L * 128;
  CUtensorMap mq, mk, mv;
  int rc;
  // time mode: Q in 128-row boxes, K and V in 64-row key tiles
  const uint32_t kvbox[3] = {box[0], mode == 0 ? 64u : box[1], box[2]};
  if ((rc = make_map_cached(h, &mq, Q, 3, dims, strides, box)) || (rc = make_map_cached(h, &mk, K, 3, dims, strides, kvbox)) ||
      (rc = make_map_cached(h, &mv, V, 3, dims, strides, kvbox)))
    return rc;
  return check_launch(trc::launch_attention(h->prec, mq, mk, mv, a, h->num_sms, st), "attention");
}

// Models whose width D is not 256: Y = A W^T (+ b) in fp32 through EPI_F32, then X += Y and
// xn = X / max(|X|, 1e-12) by the row kernel (the unfused gemm + add_rmsnorm pair of kernels.cpp:543-586).
int run_res_add(trc_handle* h, int layer, int which, const void* A, float* X, void* xn, int64_t rows, cudaStream_t st) {
  LayerDev& lw = *h->layers[layer];
  const int k = which == 0 ? 512 : h->ff;
  const int D = h->dim;
  CUtensorMap ma, mo[3];
  int rc = map_2d_cached(h, &ma, A, (uint64_t)k, (uint64_t)rows, 128);
  if (rc) return rc;
  const uint64_t dims[2] = {(uint64_t)D, (uint64_t)rows};
  const uint64_t st_y[1] = {(uint64_t)D * 4};
  const uint32_t box_y[2] = {32, 32};
  if ((rc = make_map_cached(h, &mo[0], h->Y.p, 2, dims, st_y, box_y, kMapF32))) return rc;
  mo[1] = mo[0];
  mo[2] = mo[0];
  GemmArgs a = dense_args(h, rows, D, k);
  a.out0 = h->Y.p;
  a.bias = which == 0 ? nullptr : lw.b2.p;
  if ((rc = check_launch(
           trc::launch_gemm(trc::EPI_F32, h->prec, ma, which == 0 ? lw.m_wo : lw.m_w2, mo, a, h->num_sms, st),
           "residual-branch gemm")))
    return rc;
  trc::launch_add_rmsnorm(X, h->Y.p, xn, 0, rows, 1e-12f, h->prec, D, st);
  return check_launch(cudaGetLastError(), "add_rmsnorm");
}

int run_res_norm(trc_handle* h, int layer, int which, const void* A, float* X, void* xn, int64_t rows,
                 cudaStream_t st) {
  if (h->dim != 256) return run_res_add(h, layer, which, A, X, xn, rows, st);
  LayerDev& lw = *h->layers[layer];
  const int k = which == 0 ? 512 : h->ff;
  CUtensorMap ma;
  int rc = map_2d_cached(h, &ma, A, (uint64_t)k, (uint64_t)rows, 128);
  if (rc) return rc;
  GemmArgs a = dense_args(h, rows, 256, k);
  a.out0 = X;
  a.out1 = xn;
  a.bias = which == 0 ? nullptr : lw.b2.p;
  // X (fp32) and xn (16-bit) move through TMA in boxes of 32 rows: 32 columns of X, 64 of xn
  CUtensorMap mo[3];
  const uint64_t dims[2] = {256, (uint64_t)rows};
  const uint64_t st_x[1] = {256 * 4}, st_n[1] = {256 * 2};
  const uint32_t box_x[2] = {32, 32}, box_n[2] = {64, 32};
  if ((rc = make_map_cached(h, &mo[0], X, 2, dims, st_x, box_x, kMapF32))) return rc;
  if ((rc = make_map_cached(h, &mo[1], xn, 2, dims, st_n, box_n))) return rc;
  mo[2] = mo[1];
  return check_launch(
      trc::launch_gemm(trc::EPI_RESNORM, h->prec, ma, which == 0 ? lw.m_wo : lw.m_w2, mo, a, h->num_sms, st),
      "res-norm gemm");
}

// Fused feed-forward block: X += GELU(xn W1^T + b1) W2^T + b2, xn_out = X / max(|X|, 1e-12) (mlp.cuh).
// xn_out may be xn itself: a row block's output is written after every read of that block's input.
int run_gelu(trc_handle* h, int layer, const void* xn, void* H, int64_t rows, cudaStream_t st);

int run_ffn(trc_handle* h, int layer, const void* xn, float* X, void* xn_out, int64_t rows, cudaStream_t st) {
  LayerDev& lw = *h->layers[layer];
  if (h->dim != 256) {  // unfused: H = GELU(xn W1^T + b1), then the residual branch H W2^T + b2
    int rc = run_gelu(h, layer, xn, h->H.p, rows, st);
    if (rc) return rc;
    return run_res_add(h, layer, 1, h->H.p, X, xn_out, rows, st);
  }
  if (h->ff % 128) return fail(TRC_E_INVALID, "the fused feed-forward needs a hidden width that is a multiple of 128");
  CUtensorMap ma, mx, mxn;
  int rc;
  if ((rc = map_2d_cached(h, &ma, xn, 256, (uint64_t)rows, 128))) return rc;
  const uint64_t dims[2] = {256, (uint64_t)rows};
  const uint64_t st_x[1] = {256 * 4}, st_n[1] = {256 * 2};
  const uint32_t box_x[2] = {32, 32}, box_n[2] = {64, 32};
  if ((rc = make_map_cached(h, &mx, X, 2, dims, st_x, box_x, kMapF32))) return rc;
  if ((rc = make_map_cached(h, &mxn, xn_out, 2, dims, st_n, box_n))) return rc;
  trc::MlpArgs a;
  a.num_blocks = (int)((rows + 127) / 128);
  a.M = (int)rows;
  a.n_chunks = h->ff / 128;
  a.b1 = lw.b1.p;
  a.b2 = lw.b2.p;
  a.eps = 1e-12f;
  a.err = h->err.p;
  return check_launch(trc::launch_mlp(h->prec, ma, lw.m_w1c, lw.m_w2, mx, mxn, a, h->num_sms, st), "feed-forward");
}

int run_gelu(trc_handle* h, int layer, const void* xn, void* H, int64_t rows, cudaStream_t st) {
  LayerDev& lw = *h->layers[layer];
  CUtensorMap ma;
  int rc = map_2d_cached(h, &ma, xn, (uint64_t)h->dim, (uint64_t)rows, 128);
  if (rc) return rc;
  CUtensorMap mo[3];
  if ((rc = map_2d_cached(h, &mo[0], H, (uint64_t)h->ff, (uint64_t)rows, 128))) return rc;
  mo[1] = mo[0];
  mo[2] = mo[0];
  GemmArgs a = dense_args(h, rows, h->ff, h->dim);
  a.out0 = H;
  a.bias = lw.b1.p;
  a.ld_out = h->ff;
  return check_launch(trc::launch_gemm(trc::EPI_GELU, h->prec, ma, lw.m_w1, mo, a, h->num_sms, st), "gelu gemm");
}

int run_mask(trc_handle* h, const void* xn, int B, int T, float* mask, void* hid, cudaStream_t st) {
  const int F = h->nb;
  const int BT = B * T;
  const int mt = (BT + 127) / 128;
  int rc;
  // layer 1: per band, tanh(xn_band W1'^T + b1) -> hid [band][BT][hidden]
  {
    CUtensorMap ma;
    const uint64_t dims[3] = {(uint64_t)h->dim, (uint64_t)F, (uint64_t)BT};
    const uint64_t strides[2] = {(uint64_t)h->dim * 2, (uint64_t)F * h->dim * 2};
    const uint32_t box[3] = {64, 1, 128};
    if ((rc = make_map_cached(h, &ma, xn, 3, dims, strides, box))) return rc;
    CUtensorMap mo[3];
    {
      const uint64_t odims[3] = {(uint64_t)h->hidden, (uint64_t)BT, (uint64_t)F};
      const uint64_t ostr[2] = {(uint64_t)h->hidden * 2, (uint64_t)BT * h->hidden * 2};
      const uint32_t obox[3] = {64, 128, 1};
      if ((rc = make_map_cached(h, &mo[0], hid, 3, odims, ostr, obox))) return rc;
      mo[1] = mo[0];
      mo[2] = mo[0];
    }
    GemmArgs a;
    std::memset(&a, 0, sizeof(a));
    a.k_blocks = h->dim / 64;
    a.a_mode = trc::A_GROUP_ROWS;
    a.M = BT;
    a.n_groups = F;
    const int nt = (h->hidden + 255) / 256;
    int acc = 0;
    for (int g = 0; g < F; ++g) {
      a.g_tile_start[g] = acc;
      a.g_ntiles[g] = nt;
      a.g_brow[g] = g * h->hidden;
      a.g_ncols[g] = h->hidden;
      acc += mt * nt;
    }
    a.g_tile_start[F] = acc;
    a.num_tiles = acc;
    a.out0 = hid;
    a.bias = h->mk_b1.p;
    a.ld_out = h->hidden;
    a.err = h->err.p;
    if ((rc = check_launch(trc::launch_gemm(trc::EPI_MASK_TANH, h->prec, ma, h->m_mk_w1, mo, a, h->num_sms, st),
                           "mask layer 1")))
      return rc;
  }
  // layer 2 + GLU: per band, (a, g) interleaved columns -> mask [BT][width]
  {
    CUtensorMap ma;
    const uint64_t dims[3] = {(uint64_t)h->hidden, (uint64_t)BT, (uint64_t)F};
    const uint64_t strides[2] = {(uint64_t)h->hidden * 2, (uint64_t)BT * h->hidden * 2};
    const uint32_t box[3] = {64, 128, 1};
    if ((rc = make_map_cached(h, &ma, hid, 3, dims, strides, box))) return rc;
    const CUtensorMap mo[3] = {ma, ma, ma};  // unused by this epilogue
    GemmArgs a;
    std::memset(&a, 0, sizeof(a));
    a.k_blocks = h->hidden / 64;
    a.a_mode = trc::A_ROWS_GROUP;
    a.M = BT;
    a.n_groups = F;
    int acc = 0;
    for (int g = 0; g < F; ++g) {
      const int ncols = 8 * h->freqs[g];
      const int nt = (ncols + 255) / 256;
      a.g_tile_start[g] = acc;
      a.g_ntiles[g] = nt;
      a.g_brow[g] = h->m2_off[g];
      a.g_ncols[g] = ncols;
      a.g_outoff[g] = h->band_off[g];
      acc += mt * nt;
    }
    a.g_tile_start[F] = acc;
    a.num_tiles = acc;
    a.out0 = mask;
    a.bias = h->mk_b2.p;
    a.ld_out = h->width;
    a.err = h->err.p;
    if ((rc = check_launch(trc::launch_gemm(trc::EPI_MASK_GLU, h->prec, ma, h->m_mk_w2, mo, a, h->num_sms, st),
                           "mask layer 2")))
      return rc;
  }
  return TRC_OK;
}

int frames_for(const trc_handle* h, int64_t samples) { return (int)(1 + samples / h->hop); }

// Band split for models whose width D is not 256: the grouped GEMM writes X = A W'^T + b through EPI_F32
// (ceil(D / 256) column tiles per band), then the row kernel makes xn.
int run_band_split_wide(trc_handle* h, const CUtensorMap& ma, int rows, float* X, void* xn, cudaStream_t st) {
  const int nb = h->nb, D = h->dim;
  CUtensorMap mo[3];
  const uint64_t dims[3] = {(uint64_t)D, (uint64_t)nb, (uint64_t)rows};
  const uint64_t st_x[2] = {(uint64_t)D * 4, (uint64_t)nb * D * 4};
  const uint32_t box_x[3] = {32, 1, 32};
  int rc;
  if ((rc = make_map_cached(h, &mo[0], X, 3, dims, st_x, box_x, kMapF32))) return rc;
  mo[1] = mo[0];
  mo[2] = mo[0];
  GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.a_mode = trc::A_BAND;
  a.M = rows;
  a.F = nb;
  a.n_groups = nb;
  const int mt = (rows + 127) / 128, nt = (D + 255) / 256;
  for (int g = 0; g < nb; ++g) {
    a.g_tile_start[g] = g * mt * nt;
    a.g_ntiles[g] = nt;
    a.g_brow[g] = 0;
    a.g_ncols[g] = D;
    a.g_koff[g] = h->pad_off[g];
    a.g_kblocks[g] = (h->pad_off[g + 1] - h->pad_off[g]) / 64;
  }
  a.g_tile_start[nb] = nb * mt * nt;
  a.num_tiles = nb * mt * nt;
  a.out0 = X;
  a.bias = h->bs_bias.p;
  a.bias_gstride = D;
  a.err = h->err.p;
  if ((rc = check_launch(trc::launch_gemm(trc::EPI_F32, h->prec, ma, h->m_bs_w, mo, a, h->num_sms, st), "band split")))
    return rc;
  trc::launch_rownorm(X, xn, (int64_t)rows * nb, 1e-12f, h->prec, D, st);
  return check_launch(cudaGetLastError(), "norm");
}

// Band split (model.py:147-155) + the transformers' first norm: the band-pack kernel normalises and pads
// each band's inputs into h->bs_a (16-bit), then one grouped GEMM over the bands writes X = A W'^T + b
// [rows][nb][256] fp32 and xn = X / max(|X|, 1e-12) (16-bit).
int run_band_split(trc_handle* h, const float* xin, int B, int T, float* X, void* xn, cudaStream_t st) {
  const int rows = B * T;
  const int nb = h->nb;
  trc::launch_band_pack(xin, h->width, rows, nb, h->bs_off.p, h->bs_poff.p, h->bs_kp, h->bs_a.p, h->prec, st);
  int rc;
  if ((rc = check_launch(cudaGetLastError(), "band pack"))) return rc;
  CUtensorMap ma;
  if ((rc = map_2d_cached(h, &ma, h->bs_a.p, h->bs_kp, rows, 128))) return rc;
  if (h->dim != 256) return run_band_split_wide(h, ma, rows, X, xn, st);
  // X (fp32) and xn (16-bit) as 3-D views (256, bands, rows), stored by TMA in boxes of 32 rows of one
  // band: 32 columns of X, 64 of xn
  CUtensorMap mo[3];
  {
    const uint64_t dims[3] = {256, (uint64_t)nb, (uint64_t)rows};
    const uint64_t st_x[2] = {256 * 4, (uint64_t)nb * 256 * 4}, st_n[2] = {256 * 2, (uint64_t)nb * 256 * 2};
    const uint32_t box_x[3] = {32, 1, 32}, box_n[3] = {64, 1, 32};
    if ((rc = make_map_cached(h, &mo[0], X, 3, dims, st_x, box_x, kMapF32))) return rc;
    if ((rc = make_map_cached(h, &mo[1], xn, 3, dims, st_n, box_n))) return rc;
    mo[2] = mo[1];
  }
  GemmArgs a;
  std::memset(&a, 0, sizeof(a));
  a.a_mode = trc::A_BAND;
  a.M = rows;
  a.F = nb;
  a.n_groups = nb;
  const int mt = (rows + 127) / 128;
  for (int g = 0; g < nb; ++g) {
    a.g_tile_start[g] = g * mt;
    a.g_ntiles[g] = 1;
    a.g_brow[g] = 0;
    a.g_ncols[g] = 256;
    a.g_koff[g] = h->pad_off[g];
    a.g_kblocks[g] = (h->pad_off[g + 1] - h->pad_off[g]) / 64;
  }
  a.g_tile_start[nb] = nb * mt;
  a.num_tiles = nb * mt;
  a.out0 = X;
  a.out1 = xn;
  a.bias = h->bs_bias.p;
  a.eps = 1e-12f;
  a.err = h->err.p;
  return check_launch(trc::launch_gemm(trc::EPI_BAND, h->prec, ma, h->m_bs_w, mo, a, h->num_sms, st), "band split");
}

// The 2*depth transformers of fast.py:269-341 on the residual stream X [batch*T*bands][256] fp32 (updated
// in place): the first norm, then per transformer qkv + rotary, attention, out-projection + residual +
// norm, feed-forward + residual + norm (xn_ready: h->xn already holds the first norm). The last normalised
// stream is left in h->xn (the mask's input).
int run_transformers(trc_handle* h, float* X, int batch, int T, cudaStream_t st, bool xn_ready) {
  const int64_t rows = (int64_t)batch * T * h->nb;
  int rc;
  if (!xn_ready) {
    {
      Section sec(h, "norm", st);
      trc::launch_rownorm(X, h->xn.p, rows, 1e-12f, h->prec, h->dim, st);
    }
    if ((rc = check_launch(cudaGetLastError(), "norm"))) return rc;
  }
  for (int l = 0; l < 2 * h->depth; ++l) {
    const int mode = l & 1;
    {
      Section sec(h, "qkv_rope_gemm", st);
      if ((rc = run_qkv(h, l, h->xn.p, batch, T, h->Q.p, h->K.p, h->V.p, h->G.p, st))) return rc;
    }
    {
      Section sec(h, mode == 0 ? "attention_t" : "attention_f", st);
      if ((rc = run_attention(h, mode, h->Q.p, h->K.p, h->V.p, h->G.p, h->O.p, batch, T, st))) return rc;
    }
    {
      Section sec(h, "gemm_out_res_norm", st);
      if ((rc = run_res_norm(h, l, 0, h->O.p, X, h->xn.p, rows, st))) return rc;
    }
    {
      Section sec(h, "ffn_res_norm", st);
      if ((rc = run_ffn(h, l, h->xn.p, X, h->xn.p, rows, st))) return rc;
    }
  }
  return TRC_OK;
}

}  // namespace

// ================================================================================================ C ABI
extern "C" {

const char* trc_last_error(void) { return g_last_error.c_str(); }

int trc_create(const trc_config* cfg, int device, trc_handle** out) {
  if (!cfg || !out) return fail(TRC_E_INVALID, "null argument");
  *out = nullptr;
  if (cfg->dim % 64 || cfg->dim < 128 || cfg->dim > 1024)
    return fail(TRC_E_INVALID, "dim must be a multiple of 64 in [128, 1024]");
  if (cfg->heads != 8 || cfg->dim_head != 64) return fail(TRC_E_INVALID, "only heads=8, dim_head=64 is supported");
  if (cfg->depth < 1) return fail(TRC_E_INVALID, "depth must be >= 1");
  const int n = cfg->n_fft;
  if (n < 256 || n > 4096 || (n & (n - 1))) return fail(TRC_E_INVALID, "n_fft must be a power of two in [256, 4096]");
  if (cfg->win_length != n) return fail(TRC_E_INVALID, "win_length must equal n_fft");
  if (cfg->hop < 1) return fail(TRC_E_INVALID, "hop must be >= 1");
  if (cfg->n_bands < 1 || cfg->n_bands > 64 || !cfg->freqs_per_band)
    return fail(TRC_E_INVALID, "n_bands must be in [1, 64]");
  if (cfg->ff_mult < 1) return fail(TRC_E_INVALID, "bad ff_mult");
  if (cfg->mlp_expansion_factor < 1) return fail(TRC_E_INVALID, "bad mlp_expansion_factor");
  if (cfg->precision != TRC_PREC_FP16 && cfg->precision != TRC_PREC_BF16)
    return fail(TRC_E_INVALID, "precision must be TRC_PREC_FP16 or TRC_PREC_BF16");
  int total = 0;
  for (int i = 0; i < cfg->n_bands; ++i) {
    if (cfg->freqs_per_band[i] < 1) return fail(TRC_E_INVALID, "band widths must be >= 1");
    total += cfg->freqs_per_band[i];
  }
  if (total != n / 2 + 1) return fail(TRC_E_INVALID, "freqs_per_band must sum to n_fft/2+1 = %d", n / 2 + 1);
  int ndev = 0;
  TRC_CUDA(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(TRC_E_INVALID, "device %d out of range (%d devices)", device, ndev);
  TRC_CUDA(cudaSetDevice(device));
  int major = 0, minor = 0;
  TRC_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device));
  TRC_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device));
  if (major != 10 || minor != 0)
    return fail(TRC_E_INVALID, "device %d is sm_%d%d; this library is built for sm_100a (B200)", device, major, minor);
  auto h = std::make_unique<trc_handle>();
  h->device = device;
  TRC_CUDA(cudaDeviceGetAttribute(&h->num_sms, cudaDevAttrMultiProcessorCount, device));
  h->depth = cfg->depth;
  h->dim = cfg->dim;
  h->ff = cfg->dim * cfg->ff_mult;
  h->hidden = cfg->dim * cfg->mlp_expansion_factor;
  if (h->ff % 256 || h->hidden % 256) return fail(TRC_E_INVALID, "ff and mask hidden widths must be multiples of 256");
  h->nb = cfg->n_bands;
  h->n_fft = n;
  h->hop = cfg->hop;
  h->prec = cfg->precision;
  h->freqs.assign(cfg->freqs_per_band, cfg->freqs_per_band + cfg->n_bands);
  h->band_off.assign(h->nb + 1, 0);
  h->m2_off.assign(h->nb + 1, 0);
  for (int i = 0; i < h->nb; ++i) {
    h->band_off[i + 1] = h->band_off[i] + 4 * h->freqs[i];
    h->m2_off[i + 1] = h->m2_off[i] + 8 * h->freqs[i];
  }
  h->width = 4 * (n / 2 + 1);
  int rc = h->err.alloc(1);
  if (rc) return rc;
  TRC_CUDA(cudaMemset(h->err.p, 0, sizeof(int)));
  *out = h.release();
  return TRC_OK;
}

int trc_set_param(trc_handle* h, const char* name, const float* data, int64_t numel) {
  if (!h || !name || (!data && numel > 0) || numel < 0) return fail(TRC_E_INVALID, "null argument");
  h->params[name].assign(data, data + numel);
  h->prepared = false;
  return TRC_OK;
}

int trc_prepare(trc_handle* h) {
  if (!h) return fail(TRC_E_INVALID, "null handle");
  TRC_CUDA(cudaSetDevice(h->device));
  const int d = h->dim, ff = h->ff, prec = h->prec;
  const float sqrt_d = (float)std::sqrt((double)d);  // 16 exactly for the 256-wide models
  int rc;
  h->layers.clear();
  for (int i = 0; i < h->depth; ++i) {
    for (int j = 0; j < 2; ++j) {
      const std::string p = "layers." + std::to_string(i) + "." + std::to_string(j) + ".layers.0.";
      const auto* freqs = param(h, p + "0.rotary_embed.freqs", 32);
      const auto* ga = param(h, p + "0.norm.gamma", d);
      const auto* wqkv = param(h, p + "0.to_qkv.weight", (size_t)1536 * d);
      const auto* wg = param(h, p + "0.to_gates.weight", (size_t)8 * d);
      const auto* bg = param(h, p + "0.to_gates.bias", 8);
      const auto* wo = param(h, p + "0.to_out.0.weight", (size_t)d * 512);
      const auto* gf = param(h, p + "1.net.0.gamma", d);
      const auto* w1 = param(h, p + "1.net.1.weight", (size_t)ff * d);
      const auto* b1 = param(h, p + "1.net.1.bias", ff);
      const auto* w2 = param(h, p + "1.net.4.weight", (size_t)d * ff);
      const auto* b2 = param(h, p + "1.net.4.bias", d);
      if (!freqs || !ga || !wqkv || !wg || !bg || !wo || !gf || !w1 || !b1 || !w2 || !b2) return TRC_E_INVALID;
      if (i == 0) h->rot_freqs[j] = *freqs;  // one rotary module per axis (fast.py:135-137)
      // fast.py:165-170: W_qkv * (gamma * sqrt(d)), q rows * 1/8 (exact), gates the same; fused 1544 rows
      std::vector<float> wf((size_t)1544 * d);
      std::vector<float> g(d);
      for (int c = 0; c < d; ++c) g[c] = (*ga)[c] * sqrt_d;
      for (int o = 0; o < 1536; ++o)
        for (int c = 0; c < d; ++c) {
          float v = (*wqkv)[(size_t)o * d + c] * g[c];
          if (o < 512) v *= 0.125f;
          wf[(size_t)o * d + c] = v;
        }
      for (int o = 0; o < 8; ++o)
        for (int c = 0; c < d; ++c) wf[(size_t)(1536 + o) * d + c] = (*wg)[(size_t)o * d + c] * g[c];
      // fast.py:172-181: W1 * (gamma_ff * sqrt(d))
      std::vector<float> w1f((size_t)ff * d);
      for (int c = 0; c < d; ++c) g[c] = (*gf)[c] * sqrt_d;
      for (int o = 0; o < ff; ++o)
        for (int c = 0; c < d; ++c) w1f[(size_t)o * d + c] = (*w1)[(size_t)o * d + c] * g[c];
      auto L = std::make_unique<LayerDev>();
      if ((rc = upload_bits(L->wqkv, wf, prec)) || (rc = L->gbias.upload(*bg)) || (rc = upload_bits(L->wo, *wo, prec)) ||
          (rc = upload_bits(L->w1, w1f, prec)) || (rc = L->b1.upload(*b1)) || (rc = upload_bits(L->w2, *w2, prec)) ||
          (rc = L->b2.upload(*b2)))
        return rc;
      if ((rc = map_2d(&L->m_wqkv, prec, L->wqkv.p, d, 1544, 256)) || (rc = map_2d(&L->m_wo, prec, L->wo.p, 512, d, 256)) ||
          (rc = map_2d(&L->m_w1, prec, L->w1.p, d, ff, 256)) || (rc = map_2d(&L->m_w2, prec, L->w2.p, ff, d, 256)) ||
          (rc = map_2d(&L->m_w1c, prec, L->w1.p, d, ff, 128)))
        return rc;
      h->layers.push_back(std::move(L));
    }
  }
  // band split (model.py:147-155) as one grouped GEMM over the bands: W' [256][bs_kp] 16-bit with the
  // RMSNorm gain sqrt(din) * gamma folded in, band k in columns [pad_off[k], pad_off[k] + din) and zeros
  // up to the next multiple of 64; bias [nb][256]
  {
    h->pad_off.assign(h->nb + 1, 0);
    for (int k = 0; k < h->nb; ++k) h->pad_off[k + 1] = h->pad_off[k] + (4 * h->freqs[k] + 63) / 64 * 64;
    h->bs_kp = h->pad_off[h->nb];
    const int kp = h->bs_kp;
    std::vector<float> w((size_t)d * kp, 0.f), bias((size_t)h->nb * d);
    for (int k = 0; k < h->nb; ++k) {
      const int din = 4 * h->freqs[k];
      const std::string p = "band_split.to_features." + std::to_string(k) + ".";
      const auto* gk = param(h, p + "0.gamma", din);
      const auto* wk = param(h, p + "1.weight", (size_t)d * din);
      const auto* bk = param(h, p + "1.bias", d);
      if (!gk || !wk || !bk) return TRC_E_INVALID;
      const float sc = (float)std::sqrt((double)din);
      for (int o = 0; o < d; ++o)
        for (int c = 0; c < din; ++c) w[(size_t)o * kp + h->pad_off[k] + c] = (*wk)[(size_t)o * din + c] * (sc * (*gk)[c]);
      for (int o = 0; o < d; ++o) bias[(size_t)k * d + o] = (*bk)[o];
    }
    if ((rc = upload_bits(h->bs_w, w, prec)) || (rc = h->bs_bias.upload(bias)) || (rc = h->bs_off.upload(h->band_off)) ||
        (rc = h->bs_poff.upload(h->pad_off)) || (rc = map_2d(&h->m_bs_w, prec, h->bs_w.p, kp, d, 256)))
      return rc;
  }
  // mask estimator (model.py:158-178; fast.py:140-160, 385-386): final gain folded into layer 1,
  // layer-2 rows interleaved as (a_c, g_c) pairs so the GLU is thread-local.
  {
    const auto* fg = param(h, "final_norm.gamma", d);
    if (!fg) return TRC_E_INVALID;
    const int hid = h->hidden;
    std::vector<float> g(d);
    for (int c = 0; c < d; ++c) g[c] = (*fg)[c] * sqrt_d;
    std::vector<float> w1((size_t)h->nb * hid * d), b1((size_t)h->nb * hid);
    std::vector<float> w2((size_t)h->m2_off[h->nb] * hid), b2((size_t)h->m2_off[h->nb]);
    for (int k = 0; k < h->nb; ++k) {
      const int din = 4 * h->freqs[k];
      const std::string p = "mask_estimators.0.to_freqs." + std::to_string(k) + ".0.";
      const auto* a1 = param(h, p + "0.weight", (size_t)hid * d);
      const auto* c1 = param(h, p + "0.bias", hid);
      const auto* a2 = param(h, p + "2.weight", (size_t)2 * din * hid);
      const auto* c2 = param(h, p + "2.bias", 2 * din);
      if (!a1 || !c1 || !a2 || !c2) return TRC_E_INVALID;
      for (int o = 0; o < hid; ++o) {
        for (int c = 0; c < d; ++c) w1[((size_t)k * hid + o) * d + c] = (*a1)[(size_t)o * d + c] * g[c];
        b1[(size_t)k * hid + o] = (*c1)[o];
      }
      const int r0 = h->m2_off[k];
      for (int c = 0; c < din; ++c) {
        for (int e = 0; e < 2; ++e) {
          const int src = e * din + c;  // e = 0: value half, e = 1: gate half (GLU, dim=-1)
          const size_t dst = (size_t)r0 + 2 * c + e;
          std::memcpy(&w2[dst * hid], &(*a2)[(size_t)src * hid], sizeof(float) * hid);
          b2[dst] = (*c2)[src];
        }
      }
    }
    if ((rc = upload_bits(h->mk_w1, w1, prec)) || (rc = h->mk_b1.upload(b1)) || (rc = upload_bits(h->mk_w2, w2, prec)) ||
        (rc = h->mk_b2.upload(b2)))
      return rc;
    if ((rc = map_2d(&h->m_mk_w1, prec, h->mk_w1.p, d, (uint64_t)h->nb * hid, 256)) ||
        (rc = map_2d(&h->m_mk_w2, prec, h->mk_w2.p, hid, (uint64_t)h->m2_off[h->nb], 256)))
      return rc;
  }
  // STFT tables: periodic Hann window (torch.hann_window), twiddles exp(-+ 2 pi i k / N)
  {
    const int n = h->n_fft;
    std::vector<float> w(n);
    for (int k = 0; k < n; ++k) w[k] = (float)(0.5 - 0.5 * std::cos(2.0 * M_PI * k / n));
    std::vector<float2> tf(n / 2), ti(n / 2);
    for (int k = 0; k < n / 2; ++k) {
      const double a = 2.0 * M_PI * k / n;
      tf[k] = make_float2((float)std::cos(a), (float)-std::sin(a));
      ti[k] = make_float2((float)std::cos(a), (float)std::sin(a));
    }
    if ((rc = h->window.upload(w)) || (rc = h->tw_fwd.upload(tf)) || (rc = h->tw_inv.upload(ti))) return rc;
  }
  h->tables.clear();
  h->params.clear();  // host copies are no longer needed
  h->prepared = true;
  return TRC_OK;
}

void trc_destroy(trc_handle* h) {
  if (!h) return;
  cudaSetDevice(h->device);
  delete h;
}

int64_t trc_output_length(const trc_handle* h, int64_t samples) {
  if (!h || h->hop <= 0) return -1;
  return (int64_t)h->hop * (samples / h->hop);
}

int trc_check(trc_handle* h, void* stream) {
  if (!h) return fail(TRC_E_INVALID, "null handle");
  TRC_CUDA(cudaSetDevice(h->device));
  TRC_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
  int e = 0;
  TRC_CUDA(cudaMemcpy(&e, h->err.p, sizeof(int), cudaMemcpyDeviceToHost));
  if (e != 0) {
    TRC_CUDA(cudaMemset(h->err.p, 0, sizeof(int)));
    return fail(TRC_E_DEVICE, "device error %d reported by a kernel (bounded wait expired or bad arguments)", e);
  }
  return TRC_OK;
}

int trc_error_async(trc_handle* h, int* host_word, void* stream) {
  if (!h || !host_word) return fail(TRC_E_INVALID, "null handle or host word");
  TRC_CUDA(cudaSetDevice(h->device));
  cudaStream_t st = (cudaStream_t)stream;
  TRC_CUDA(cudaMemcpyAsync(host_word, h->err.p, sizeof(int), cudaMemcpyDeviceToHost, st));
  TRC_CUDA(cudaMemsetAsync(h->err.p, 0, sizeof(int), st));
  return TRC_OK;
}

int trc_selftest_wait_timeout(trc_handle* h, void* stream) {
  if (!h) return fail(TRC_E_INVALID, "null handle");
  TRC_CUDA(cudaSetDevice(h->device));
  trc::launch_wait_timeout_selftest(h->err.p, (cudaStream_t)stream);
  return check_launch(cudaGetLastError(), "wait-timeout self-test");
}

#define TRC_REQUIRE_PREPARED(h)                                               \
  do {                                                                        \
    if (!(h)) return fail(TRC_E_INVALID, "null handle");                      \
    if (!(h)->prepared) return fail(TRC_E_STATE, "trc_prepare has not run"); \
    TRC_CUDA(cudaSetDevice((h)->device));                                     \
  } while (0)

int trc_forward(trc_handle* h, const float* d_audio, int batch, int64_t samples, float* d_out, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (!d_audio || !d_out || batch < 1) return fail(TRC_E_INVALID, "bad forward arguments");
  if (samples <= h->n_fft / 2) return fail(TRC_E_INVALID, "samples must exceed n_fft/2 = %d", h->n_fft / 2);
  const int T = frames_for(h, samples);
  if ((int64_t)batch * T * h->nb >= (1ll << 31) / 512) return fail(TRC_E_INVALID, "batch too large");
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if ((rc = ensure_workspace(h, batch, T))) return rc;
  {
    Section sec(h, "stft", st);
    trc::launch_stft(d_audio, batch, samples, T, h->n_fft, h->hop, h->window.p, h->tw_fwd.p, h->xin.p, st);
  }
  if ((rc = check_launch(cudaGetLastError(), "stft"))) return rc;
  {
    Section sec(h, "band_split", st, 2);
    if ((rc = run_band_split(h, h->xin.p, batch, T, h->X.p, h->xn.p, st))) return rc;
  }
  if ((rc = run_transformers(h, h->X.p, batch, T, st, true))) return rc;
  {
    Section sec(h, "mask", st, 2);
    if ((rc = run_mask(h, h->xn.p, batch, T, h->mask.p, h->H.p, st))) return rc;
  }
  {
    Section sec(h, "istft", st, 2);
    trc::launch_istft(h->xin.p, h->mask.p, batch, T, h->n_fft, h->hop, h->window.p, h->tw_inv.p, h->frames.p, d_out,
                      st);
  }
  return check_launch(cudaGetLastError(), "istft");
}

int trc_transformer(trc_handle* h, float* d_X, int batch, int T, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (!d_X || batch < 1 || T < 1) return fail(TRC_E_INVALID, "bad transformer arguments");
  if ((int64_t)batch * T * h->nb >= (1ll << 31) / 512) return fail(TRC_E_INVALID, "batch too large");
  int rc;
  if ((rc = ensure_workspace(h, batch, T))) return rc;
  return run_transformers(h, d_X, batch, T, (cudaStream_t)stream, false);
}

int trc_profile(trc_handle* h, int enable) {
  if (!h) return fail(TRC_E_INVALID, "null handle");
  TRC_CUDA(cudaSetDevice(h->device));
  TRC_CUDA(cudaDeviceSynchronize());
  for (auto& p : h->ev_pending) {
    h->ev_pool.push_back(p.second.first);
    h->ev_pool.push_back(p.second.second);
  }
  h->ev_pending.clear();
  h->section.clear();
  h->timing = enable != 0;
  // create the events up front so the timed region does not pay for cudaEventCreate
  while (h->timing && h->ev_pool.size() < 4096) {
    cudaEvent_t e = nullptr;
    TRC_CUDA(cudaEventCreate(&e));
    h->ev_pool.push_back(e);
  }
  return TRC_OK;
}

int trc_profile_read(trc_handle* h, char* buf, int buflen) {
  if (!h || !buf || buflen < 1) return fail(TRC_E_INVALID, "bad profile_read arguments");
  TRC_CUDA(cudaSetDevice(h->device));
  for (auto& p : h->ev_pending) {
    TRC_CUDA(cudaEventSynchronize(p.second.second));
    float ms = 0.f;
    TRC_CUDA(cudaEventElapsedTime(&ms, p.second.first, p.second.second));
    h->section[p.first].first += ms;
    h->ev_pool.push_back(p.second.first);
    h->ev_pool.push_back(p.second.second);
  }
  h->ev_pending.clear();
  std::string out;
  char line[160];
  for (auto& kv : h->section) {
    snprintf(line, sizeof(line), "%s %.6f %ld\n", kv.first.c_str(), kv.second.first, kv.second.second);
    out += line;
  }
  if ((int)out.size() + 1 > buflen) return fail(TRC_E_INVALID, "profile buffer too small (%zu bytes needed)", out.size() + 1);
  std::memcpy(buf, out.c_str(), out.size() + 1);
  return TRC_OK;
}

long long trc_launch_count(void) { return g_launches.load(); }

// Symmetric Hamming window of `chunk` samples in float64 rounded to float32 (chunking.py:24-28), made
// and uploaded once per (device, length) and kept for the life of the process: a per-call upload of
// megabytes from pageable memory would wait for the stream to drain (the staging buffers only empty
// as the stream reaches the copy), which stalls the host behind a whole song of queued work.
static int hamming_cached(int64_t chunk, const float** out) {
  static std::mutex mu;
  static std::map<std::pair<int, int64_t>, float*> cache;
  int dev = 0;
  TRC_CUDA(cudaGetDevice(&dev));
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find({dev, chunk});
  if (it != cache.end()) {
    *out = it->second;
    return TRC_OK;
  }
  std::vector<float> w((size_t)chunk);
  if (chunk == 1) {
    w[0] = 1.0f;
  } else {
    for (int64_t k = 0; k < chunk; ++k) w[k] = (float)(0.54 - 0.46 * std::cos(2.0 * M_PI * (double)k / (double)(chunk - 1)));
  }
  float* d = nullptr;
  TRC_CUDA(cudaMalloc(&d, sizeof(float) * chunk));
  if (cudaError_t e = cudaMemcpy(d, w.data(), sizeof(float) * chunk, cudaMemcpyHostToDevice); e != cudaSuccess) {
    cudaFree(d);  // not cached: the next call retries
    return fail(TRC_E_CUDA, "Hamming window upload failed: %s", cudaGetErrorString(e));
  }
  cache[{dev, chunk}] = d;
  *out = d;
  return TRC_OK;
}

int trc_ola(const float* d_chunks, int64_t chunk_out_len, const int64_t* h_starts, int n_chunks, int64_t chunk,
            int64_t n, float* d_result, void* stream) {
  if (!d_chunks || !h_starts || !d_result || n_chunks < 1 || chunk < 1 || n < 1 || chunk_out_len < 1 ||
      chunk_out_len > chunk)
    return fail(TRC_E_INVALID, "bad overlap-add arguments");
  for (int i = 0; i < n_chunks; ++i) {
    if (h_starts[i] < 0 || h_starts[i] + chunk > n) return fail(TRC_E_INVALID, "chunk %d out of range", i);
    if (i && h_starts[i] <= h_starts[i - 1]) return fail(TRC_E_INVALID, "starts must be increasing");
  }
  cudaStream_t st = (cudaStream_t)stream;
  const float* d_w = nullptr;
  if (int rc = hamming_cached(chunk, &d_w)) return rc;
  // the starts are a few hundred bytes: a pageable copy is staged at once and never waits on the stream
  int64_t* d_s = nullptr;
  TRC_CUDA(cudaMallocAsync(&d_s, sizeof(int64_t) * n_chunks, st));
  if (cudaError_t e = cudaMemcpyAsync(d_s, h_starts, sizeof(int64_t) * n_chunks, cudaMemcpyHostToDevice, st);
      e != cudaSuccess) {
    cudaFreeAsync(d_s, st);
    return fail(TRC_E_CUDA, "chunk starts upload failed: %s", cudaGetErrorString(e));
  }
  trc::launch_chunk_ola(d_chunks, chunk_out_len, d_s, n_chunks, d_w, n, d_result, st);
  g_launches += 1;
  cudaError_t e = cudaGetLastError();
  TRC_CUDA(cudaFreeAsync(d_s, st));
  return check_launch(e, "overlap-add");
}

int trc_remix(const float* d_in, int channels, int64_t n, const double* h_gains, float* d_out, void* stream) {
  if (!d_in || !h_gains || !d_out || channels < 1 || channels > trc::kRemixMaxChannels || n < 1)
    return fail(TRC_E_INVALID, "bad remix arguments");
  trc::launch_remix(d_in, channels, n, h_gains, d_out, (cudaStream_t)stream);
  g_launches += 1;
  return check_launch(cudaGetLastError(), "remix");
}

int trc_resample(const float* d_in, int channels, int64_t n_in, int up, int down, int64_t half, const double* d_taps,
                 int k_per_phase, int64_t n_out, float* d_out, void* stream) {
  if (!d_in || !d_taps || !d_out || channels < 1 || channels > 65535 || n_in < 1 || n_out < 1 || up < 1 ||
      down < 1 || half < 0 || k_per_phase < 1 || (int64_t)k_per_phase * up > (int64_t)1 << 26 ||
      (n_out - 1) > (INT64_MAX - half) / down)
    return fail(TRC_E_INVALID, "bad resample arguments");
  trc::launch_resample(d_in, channels, n_in, up, down, half, d_taps, k_per_phase, n_out, d_out, (cudaStream_t)stream);
  g_launches += 1;
  return check_launch(cudaGetLastError(), "resample");
}

// ------------------------------------------------------------------------------------------------ per stage
int trc_add_rmsnorm(trc_handle* h, float* d_X, const float* d_Y, void* d_out, int out_f32, int64_t rows, float eps,
                    void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (!d_X || !d_out || rows < 0) return fail(TRC_E_INVALID, "bad add_rmsnorm arguments");
  Section sec(h, "norm", (cudaStream_t)stream);
  trc::launch_add_rmsnorm(d_X, d_Y, d_out, out_f32, rows, eps, h->prec, h->dim, (cudaStream_t)stream);
  return check_launch(cudaGetLastError(), "add_rmsnorm");
}

int trc_qkv_rope_gemm(trc_handle* h, int layer, const void* d_xn, int batch, int T, void* d_Q, void* d_K, void* d_V,
                      float* d_G, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (layer < 0 || layer >= 2 * h->depth || batch < 1 || T < 1) return fail(TRC_E_INVALID, "bad qkv arguments");
  Section sec(h, "qkv_rope_gemm", (cudaStream_t)stream);
  return run_qkv(h, layer, d_xn, batch, T, d_Q, d_K, d_V, d_G, (cudaStream_t)stream);
}

int trc_attention(trc_handle* h, int mode, const void* d_Q, const void* d_K, const void* d_V, const float* d_G,
                  void* d_O, int batch, int T, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if ((mode != 0 && mode != 1) || batch < 1 || T < 1) return fail(TRC_E_INVALID, "bad attention arguments");
  Section sec(h, mode == 0 ? "attention_t" : "attention_f", (cudaStream_t)stream);
  return run_attention(h, mode, d_Q, d_K, d_V, d_G, d_O, batch, T, (cudaStream_t)stream);
}

int trc_gemm_res_norm(trc_handle* h, int layer, int which, const void* d_A, float* d_X, void* d_xn, int64_t rows,
                      void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (layer < 0 || layer >= 2 * h->depth || (which != 0 && which != 1) || rows < 1)
    return fail(TRC_E_INVALID, "bad gemm_res_norm arguments");
  Section sec(h, which == 0 ? "gemm_out_res_norm" : "gemm_ff2_res_norm", (cudaStream_t)stream);
  return run_res_norm(h, layer, which, d_A, d_X, d_xn, rows, (cudaStream_t)stream);
}

int trc_ffn_res_norm(trc_handle* h, int layer, const void* d_xn, float* d_X, void* d_xn_out, int64_t rows,
                     void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (layer < 0 || layer >= 2 * h->depth || rows < 1 || !d_xn || !d_X || !d_xn_out)
    return fail(TRC_E_INVALID, "bad ffn_res_norm arguments");
  Section sec(h, "ffn_res_norm", (cudaStream_t)stream);
  return run_ffn(h, layer, d_xn, d_X, d_xn_out, rows, (cudaStream_t)stream);
}

int trc_gemm_gelu(trc_handle* h, int layer, const void* d_xn, void* d_H, int64_t rows, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (layer < 0 || layer >= 2 * h->depth || rows < 1) return fail(TRC_E_INVALID, "bad gemm_gelu arguments");
  Section sec(h, "gemm_ff1", (cudaStream_t)stream);
  return run_gelu(h, layer, d_xn, d_H, rows, (cudaStream_t)stream);
}

int trc_rope_pack(trc_handle* h, int mode, const void* d_qkvg, int batch, int T, void* d_Q, void* d_K, void* d_V,
                  float* d_G, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if ((mode != 0 && mode != 1) || batch < 1 || T < 1 || !d_qkvg || !d_Q || !d_K || !d_V || !d_G)
    return fail(TRC_E_INVALID, "bad rope_pack arguments");
  const int64_t N = (int64_t)batch * T * h->nb;
  if (N >= (1ll << 31)) return fail(TRC_E_INVALID, "too many tokens");
  Tables* tab = get_tables(h, mode, mode == 0 ? T : h->nb);
  if (!tab) return TRC_E_CUDA;
  Section sec(h, "rope_pack", (cudaStream_t)stream);
  trc::launch_rope_pack(h->prec, d_qkvg, tab->cos_t.p, tab->sin_t.p, mode, T, h->nb, N, d_Q, d_K, d_V, d_G,
                        (cudaStream_t)stream);
  return check_launch(cudaGetLastError(), "rope_pack");
}

int trc_gate_merge(trc_handle* h, int mode, const void* d_A, const float* d_G, void* d_O, int batch, int T,
                   void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if ((mode != 0 && mode != 1) || batch < 1 || T < 1 || !d_A || !d_G || !d_O)
    return fail(TRC_E_INVALID, "bad gate_merge arguments");
  const int64_t N = (int64_t)batch * T * h->nb;
  if (N >= (1ll << 31)) return fail(TRC_E_INVALID, "too many tokens");
  Section sec(h, "gate_merge", (cudaStream_t)stream);
  trc::launch_gate_merge(h->prec, d_A, d_G, d_O, mode, T, h->nb, N, (cudaStream_t)stream);
  return check_launch(cudaGetLastError(), "gate_merge");
}

int trc_stft(trc_handle* h, const float* d_audio, int batch, int64_t samples, float* d_xin, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (batch < 1 || samples <= h->n_fft / 2) return fail(TRC_E_INVALID, "bad stft arguments");
  const int T = frames_for(h, samples);
  Section sec(h, "stft", (cudaStream_t)stream);
  trc::launch_stft(d_audio, batch, samples, T, h->n_fft, h->hop, h->window.p, h->tw_fwd.p, d_xin, (cudaStream_t)stream);
  return check_launch(cudaGetLastError(), "stft");
}

int trc_band_split(trc_handle* h, const float* d_xin, int batch, int T, float* d_X, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (!d_xin || !d_X || batch < 1 || T < 1) return fail(TRC_E_INVALID, "bad band_split arguments");
  if ((int64_t)batch * T * h->nb >= (1ll << 31) / 512) return fail(TRC_E_INVALID, "batch too large");
  int rc;
  if ((rc = ensure_workspace(h, batch, T))) return rc;
  Section sec(h, "band_split", (cudaStream_t)stream, 2);
  return run_band_split(h, d_xin, batch, T, d_X, h->xn.p, (cudaStream_t)stream);
}

int trc_mask(trc_handle* h, const void* d_xn, int batch, int T, float* d_mask, void* d_hidden, void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (batch < 1 || T < 1 || !d_hidden || !d_xn || !d_mask) return fail(TRC_E_INVALID, "bad mask arguments");
  if (reinterpret_cast<uintptr_t>(d_mask) % 16) return fail(TRC_E_INVALID, "mask must be 16-byte aligned");
  Section sec(h, "mask", (cudaStream_t)stream, 2);
  return run_mask(h, d_xn, batch, T, d_mask, d_hidden, (cudaStream_t)stream);
}

int trc_istft(trc_handle* h, const float* d_xin, const float* d_mask, int batch, int T, float* d_out, float* d_frames,
              void* stream) {
  TRC_REQUIRE_PREPARED(h);
  if (batch < 1 || T < 2 || !d_frames) return fail(TRC_E_INVALID, "bad istft arguments");
  Section sec(h, "istft", (cudaStream_t)stream, 2);
  trc::launch_istft(d_xin, d_mask, batch, T, h->n_fft, h->hop, h->window.p, h->tw_inv.p, d_frames, d_out,
                    (cudaStream_t)stream);
  return check_launch(cudaGetLastError(), "istft");
}

}  // extern "C"
