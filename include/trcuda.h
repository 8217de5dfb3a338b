/*
 * trcuda.h - C ABI of the Blackwell (sm_100a) BS-RoFormer backend (libtrcuda.so).
 *
 * Plain C: device pointers, sizes and an opaque stream handle (a cudaStream_t passed as void*; NULL =
 * the legacy default stream). No torch types cross this boundary. Every function returns 0 on success
 * or a negative TRC_E_* code; trc_last_error() then describes the failure of the calling thread's last
 * call. Nothing here aborts the process.
 *
 * Ownership: the caller owns every device buffer it passes in; a handle owns its folded weights, its
 * tables and the work buffers of trc_forward. One forward at a time per handle (the reference's
 * Separator serialises calls with a lock, turbo_roformer/separator.py:101,226); handles on different
 * devices may be driven from different host threads.
 *
 * Devices: a function that takes a handle makes the handle's device current on the calling thread
 * (cudaSetDevice) and leaves it current on return; the caller's stream must belong to that device.
 * Functions without a handle (trc_ola, trc_ola_noalloc, trc_remix, trc_resample) run on the calling
 * thread's current device. Restoring a previous device is left to the caller, because doing so from the
 * library would create a CUDA context on a device the process may never have used.
 *
 * The reference's drop-in surface for this path is the torch op library
 *   TORCH_LIBRARY(turbo_roformer, m)          (src/turbo_roformer/csrc/kernels.cpp:644-652)
 * driven by FastBSRoformer.forward            (src/turbo_roformer/fast.py:363-394)
 * and the chunk overlap-add                   (src/turbo_roformer/chunking.py:36-61).
 * Each entry point below names the reference interface it replaces.
 *
 * 16-bit activations and weights use the handle's operand type: IEEE fp16 (TRC_PREC_FP16, default)
 * or bf16 (TRC_PREC_BF16). Accumulation, the residual stream, STFT/iSTFT, band split and the mask are fp32.
 */
#ifndef TRCUDA_H_
#define TRCUDA_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TRC_OK 0
#define TRC_E_INVALID (-1)     /* bad argument / unsupported configuration */
#define TRC_E_CUDA (-2)        /* a CUDA runtime or driver call failed */
#define TRC_E_DEVICE (-3)      /* a kernel reported a device-side error (bounded wait expired, bad args) */
#define TRC_E_STATE (-4)       /* call out of order (e.g. forward before trc_prepare) */
#define TRC_E_NOMEM (-5)       /* device allocation failed */

#define TRC_PREC_FP16 0
#define TRC_PREC_BF16 1

typedef struct trc_handle trc_handle;

/* Architecture of a single-stem stereo BS-RoFormer (turbo_roformer/model.py:181-245;
 * turbo_roformer/registry.py:49-69). Supported: dim a multiple of 64 in [128, 1024] (256 runs the fused
 * epilogue kernels; the other widths run their residual branches as fp32 GEMMs followed by row norms, as the
 * reference drops its fused kernels for them, fast.py:121-122), 8 heads x 64, depth-1 time/freq
 * transformers, mask_estimator_depth 2, power-of-two n_fft in [256, 4096] with win_length == n_fft,
 * <= 64 bands. */
typedef struct trc_config {
  int dim;
  int depth;
  int heads;
  int dim_head;
  int ff_mult;
  int n_bands;
  const int* freqs_per_band; /* n_bands entries, summing to n_fft / 2 + 1 */
  int n_fft;
  int hop;
  int win_length;
  int mlp_expansion_factor;
  int precision; /* TRC_PREC_FP16 or TRC_PREC_BF16 */
} trc_config;

/* ------------------------------------------------------------------ model lifetime
 * Replaces FastBSRoformer.__init__ + _prep (turbo_roformer/fast.py:86-191): weights are supplied by
 * their upstream state_dict key (model.py keys, e.g. "layers.0.0.layers.0.0.to_qkv.weight") as host
 * fp32 arrays; trc_prepare folds the RMSNorm gains and the 1/8 attention scale into the following
 * Linear layers, fuses qkv + gates, converts to the operand type and uploads. */
int trc_create(const trc_config* cfg, int device, trc_handle** out);
int trc_set_param(trc_handle* h, const char* name, const float* host_data, int64_t numel);
int trc_prepare(trc_handle* h);
void trc_destroy(trc_handle* h);

/* Replaces FastBSRoformer.forward (turbo_roformer/fast.py:363-394) for `batch` chunks at once:
 * d_audio [batch][2][samples] fp32 -> d_out [batch][2][hop * (samples / hop)] fp32.
 * samples must exceed n_fft / 2 (reflect padding). Asynchronous on `stream`. */
int trc_forward(trc_handle* h, const float* d_audio, int batch, int64_t samples, float* d_out, void* stream);
int64_t trc_output_length(const trc_handle* h, int64_t samples);

/* Replaces FastBSRoformer._transformer_cpp (turbo_roformer/fast.py:269-341): the 2*depth time/frequency
 * transformers alone on the fp32 residual stream d_X [batch * T * n_bands][dim] (token order
 * (batch, frame, band)), updated in place. Uses the handle's work buffers; asynchronous on `stream`. */
int trc_transformer(trc_handle* h, float* d_X, int batch, int T, void* stream);

/* Synchronises `stream` and returns TRC_E_DEVICE if a kernel of this handle recorded a device error
 * since the last check (the error word is then cleared). */
int trc_check(trc_handle* h, void* stream);

/* Non-blocking form of trc_check for callers that keep several forwards queued: enqueues on `stream` a
 * copy of the handle's device error word into *host_word (pinned host memory; valid once the stream
 * has passed this point) and then clears the device word. *host_word != 0 means a kernel queued
 * before this call on the handle recorded an error. No reference counterpart (its forward is
 * synchronous); used by Separator.submit. */
int trc_error_async(trc_handle* h, int* host_word, void* stream);

/* Self-test of the device-side failure path: launches a kernel whose bounded wait on a barrier that
 * nothing signals gives up after the wait limit (2 s) and records an error in the handle's error word,
 * which the next trc_check reports as TRC_E_DEVICE. The context and the handle stay usable. */
int trc_selftest_wait_timeout(trc_handle* h, void* stream);

/* Replaces chunking.overlap_add's accumulation (turbo_roformer/chunking.py:54-61): Hamming-weighted
 * sum of chunk outputs, divided by the summed weights (clamped at 1e-10), in start order.
 * d_chunks [n_chunks][2][chunk_out_len]; h_starts: n_chunks increasing host int64 starts; chunk = C
 * (the Hamming window length); d_result [2][n]. Bit-identical to the reference for identical chunks. */
int trc_ola(const float* d_chunks, int64_t chunk_out_len, const int64_t* h_starts, int n_chunks, int64_t chunk,
            int64_t n, float* d_result, void* stream);

const char* trc_last_error(void);

/* Replaces audio.to_stereo / downmix_stereo (turbo_roformer/audio.py:35-68) on the device:
 * d_out[o][i] = (float)(sum over k of h_gains[o * channels + k] * (double)d_in[k][i]), k ascending, fp64 with
 * separately rounded products and sums.
 * d_in [channels][n] float32; h_gains: host (2 x channels) float64 row-major, copied into the launch;
 * 1 <= channels <= 16; d_out [2][n]. */
int trc_remix(const float* d_in, int channels, int64_t n, const double* h_gains, float* d_out, void* stream);

/* Replaces audio.resample (turbo_roformer/audio.py:71-82, soxr there) on the device: polyphase FIR
 * resampling by up/down of each of `channels` rows. Output m: t = m * down + half, j0 = t / up,
 * p = t % up, d_out[c][m] = (float)(sum over k < k_per_phase of d_taps[k * up + p] * (double)d_in[c][j0 - k]),
 * inputs outside [0, n_in) being zero. d_taps [k_per_phase][up] float64 on the device: the caller's
 * filter h (odd length 2 * half + 1, gain `up` included) with d_taps[k * up + p] = h[p + k * up]. */
int trc_resample(const float* d_in, int channels, int64_t n_in, int up, int down, int64_t half, const double* d_taps,
                 int k_per_phase, int64_t n_out, float* d_out, void* stream);

/* Overlap-add that allocates nothing. No counterpart in the reference: it exists for callers that may
 * not allocate device memory while they run (an audio plugin whose host application owns all device
 * memory and forbids allocations of its own, a real-time audio thread that must not block in the
 * allocator). Same arguments, semantics and result as trc_ola, but the Hamming window and the chunk
 * starts are staged in fixed arrays inside this library (one set per GPU context that loads it, kept
 * until the process exits: TRC_OLA_NOALLOC_MAX_CHUNK floats + TRC_OLA_NOALLOC_MAX_CHUNKS int64, about
 * 8 MiB). Longer chunks or more chunks are rejected with TRC_E_INVALID. The first call in a CUDA context
 * looks the arrays up (one-time set-up); make that first call before any stream capture. The window is
 * uploaded (from pageable host memory) only when the chunk length differs from the last one uploaded in
 * that context; every call uploads its starts, 8 bytes per chunk, from pageable host memory. All calls
 * share the arrays: calls that may overlap on the GPU (different streams, or different host threads on
 * one device) race and must be serialised by the caller. */
#define TRC_OLA_NOALLOC_MAX_CHUNK (1 << 21)
#define TRC_OLA_NOALLOC_MAX_CHUNKS 8192
int trc_ola_noalloc(const float* d_chunks, int64_t chunk_out_len, const int64_t* h_starts, int n_chunks,
                    int64_t chunk, int64_t n, float* d_result, void* stream);

/* ------------------------------------------------------------------ instrumentation
 * Per-section device timing, the counterpart of the reference's opt-in per-section profile
 * (FastBSRoformer.timer, turbo_roformer/fast.py:62-80; same section keys: stft, band_split, norm,
 * qkv_rope_gemm, attention_t, attention_f, gemm_out_res_norm, gemm_ff1, gemm_ff2_res_norm, mask,
 * istft). trc_profile(h, 1) synchronises the device, clears the totals and records a CUDA event pair
 * around every section on its launch stream; trc_profile_read writes one "name total_ms launches"
 * line per section into buf (waiting for the recorded events). trc_launch_count returns the number
 * of kernels this library has launched in the process. */
int trc_profile(trc_handle* h, int enable);
int trc_profile_read(trc_handle* h, char* buf, int buflen);
long long trc_launch_count(void);

/* ------------------------------------------------------------------ per-stage entry points
 * The op-level surface of the reference (TORCH_LIBRARY(turbo_roformer), kernels.cpp:644-652), on the
 * layouts of this backend. `layer` indexes the 2*depth transformers in forward order (even = time,
 * odd = freq). Tokens are ordered (batch, frame, band): token = (b * T + t) * n_bands + f.
 * Q/K/V: [sequences][L][64] 16-bit with time sequences (b, band, head), L = T, and freq sequences
 * (b, frame, head), L = n_bands. G: [tokens][8] fp32 sigmoid gates. O: [tokens][512] 16-bit. */

/* kernels.cpp:102-137 add_rmsnorm: X (+)= Y (Y may be NULL); out = X / max(|X|, eps), rows of 256;
 * out is fp32 if out_f32 else the handle's 16-bit type. */
int trc_add_rmsnorm(trc_handle* h, float* d_X, const float* d_Y, void* d_out, int out_f32, int64_t rows, float eps,
                    void* stream);

/* kernels.cpp:442-540 qkv_rope_gemm: xn [tokens][256] -> rotary Q, K, V in the attention layout + G. */
int trc_qkv_rope_gemm(trc_handle* h, int layer, const void* d_xn, int batch, int T, void* d_Q, void* d_K, void* d_V,
                      float* d_G, void* stream);

/* kernels.cpp:255-388 attention (mode 0 = time, 1 = freq): O = merge_heads(softmax(Q K^T) V * G). */
int trc_attention(trc_handle* h, int mode, const void* d_Q, const void* d_K, const void* d_V, const float* d_G,
                  void* d_O, int batch, int T, void* stream);

/* kernels.cpp:543-586 gemm_res_norm: X += A W^T (+ b); xn = X / max(|X|, 1e-12).
 * which = 0: attention out-projection (A = O [tokens][512]); which = 1: FF2 (A = H [tokens][ff_inner]). */
int trc_gemm_res_norm(trc_handle* h, int layer, int which, const void* d_A, float* d_X, void* d_xn, int64_t rows,
                      void* stream);

/* kernels.cpp:610-642 gemm_gelu / fast.py:343-346: H = gelu(xn W1^T + b1), H [tokens][ff_inner]. */
int trc_gemm_gelu(trc_handle* h, int layer, const void* d_xn, void* d_H, int64_t rows, void* stream);

/* The reference's feed-forward pair gemm_gelu + gemm_res_norm (csrc/kernels.cpp:610-642, :543-586;
 * fast.py:320-333) in one kernel: d_X [rows][256] fp32 += GELU(d_xn W1^T + b1) W2^T + b2 and
 * d_xn_out = X / max(|X|, 1e-12) (16-bit; may equal d_xn). The hidden activation stays on chip. */
int trc_ffn_res_norm(trc_handle* h, int layer, const void* d_xn, float* d_X, void* d_xn_out, int64_t rows,
                     void* stream);

/* Replaces rope_pack (csrc/kernels.cpp:161-248, packed = false; the CPU-only VNNI packing has no GPU
 * counterpart): d_qkvg [N][1544] 16-bit output of the unfused qkv+gate GEMM (gate logits include their
 * bias) -> rotary q and k, plain v in the attention layout d_Q, d_K, d_V [seq][L][64] (16-bit) and
 * d_G [N][8] = sigmoid(gate logits) fp32. mode 0 = time (L = T), 1 = freq (L = bands); N = batch*T*bands;
 * the rotary angles are the model's (the handle's tables). */
int trc_rope_pack(trc_handle* h, int mode, const void* d_qkvg, int batch, int T, void* d_Q, void* d_K, void* d_V,
                  float* d_G, void* stream);

/* Replaces gate_merge (csrc/kernels.cpp:391-408): d_O[token][h*64 + d] = d_G[token][h] * d_A[seq][pos][d]
 * (16-bit in and out, product in fp32), the head merge of an attention computed elsewhere. */
int trc_gate_merge(trc_handle* h, int mode, const void* d_A, const float* d_G, void* d_O, int batch, int T,
                   void* stream);

/* fast.py:370-376: audio [batch][2][samples] -> spectrum xin [batch][T][n_fft/2+1][2][2] fp32. */
int trc_stft(trc_handle* h, const float* d_audio, int batch, int64_t samples, float* d_xin, void* stream);

/* model.py:147-155 via fast.py:377-380: xin -> X [tokens][256] fp32 (band split). */
int trc_band_split(trc_handle* h, const float* d_xin, int batch, int T, float* d_X, void* stream);

/* fast.py:385-387 + 349-360: xn (L2-normalised last residual, [tokens][256] 16-bit) -> mask
 * [batch][T][n_fft/2+1][2][2] fp32 (final norm gain folded into the first mask layer; d_mask 16-byte
 * aligned). d_hidden is scratch of n_bands * batch * T * dim * mlp_expansion_factor 16-bit elements. */
int trc_mask(trc_handle* h, const void* d_xn, int batch, int T, float* d_mask, void* d_hidden, void* stream);

/* fast.py:388-393: mask apply + iSTFT. xin, mask as above -> out [batch][2][hop * (T - 1)].
 * d_frames is scratch of batch * T * 2 * n_fft floats. */
int trc_istft(trc_handle* h, const float* d_xin, const float* d_mask, int batch, int T, float* d_out,
              float* d_frames, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TRCUDA_H_ */
