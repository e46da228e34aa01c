/*
 * dispatcher_b200.h — C ABI of the B200 (sm_100a) Dispatcher-Hybrid hot path.
 *
 * Plain pointers, sizes and a cudaStream_t passed as void*; no framework
 * types.  Every entry point returns 0 (DH_OK) or a DH_ERR_* code, after which
 * dh_last_error() gives a one-line message for the calling thread.  No entry
 * point allocates, synchronises the host or reads device memory on the host,
 * so all of them can be recorded into a CUDA graph; the decode position `t`
 * is read on the device from an int64 counter (`t_buf`), as the reference's
 * graphed decoder does (dispatcher_hybrid/decoding.py:361, 443).
 *
 * Layouts (row-major, bf16 = IEEE bfloat16 stored as uint16):
 *   tokens            int64 (batch)
 *   x (decode)        fp32  (batch, d)   residual stream
 *   B_hist            bf16  (batch, max_len, gh)
 *   rg_hist           bf16  (batch, max_len, L, H)
 *   V_ring            bf16  (batch, S = 2^(L+1)-2, d); ring j at slot
 *                     2^(j+1)-2, position t -> slot offset_j + (t & (2^(j+1)-1))
 *   k_cache, v_cache  bf16  (batch, max_len, H, hd); k stored after RoPE
 * Citations are to files of the reference package, dispatcher_hybrid/.
 */
#ifndef DISPATCHER_B200_H
#define DISPATCHER_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define DH_API __attribute__((visibility("default")))
#else
#define DH_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define DH_OK 0
#define DH_ERR_SHAPE 1       /* unsupported or inconsistent sizes            */
#define DH_ERR_ARG 2         /* null or misaligned pointer, bad enum value   */
#define DH_ERR_CUDA 3        /* a CUDA runtime call or launch failed         */
#define DH_ERR_TIMEOUT 4     /* a bounded device-side wait gave up           */
#define DH_ERR_DEVICE 5      /* device is not an sm_100 part                 */

/* library identity / diagnostics */
DH_API const char* dh_version(void);
DH_API const char* dh_last_error(void);
DH_API int dh_sm_count(int* out);

/* ---------------------------------------------------------------- decode */

/* x[b,:] = fp32(E[tokens[b],:]).  Replaces the embedding lookup of the
 * captured step (decoding.py:438).  Out-of-range ids are clamped and
 * reported by a nonzero *status (nullable). */
DH_API int dh_decode_embed(const int64_t* tokens, const void* emb, float* x, int batch, int d,
                    int vocab, int* status, void* stream);

/* Tree block, mixer input side (decoding.py:473-476): h = RMSNorm(x; norm_w);
 * [v0 | A | B] = h . W3^T with W3 = [W_in; W1x; W1s] (3d x d, bf16);
 * v0, A -> bf16 (batch, d); B -> B_hist[:, t, :]. */
DH_API int dh_decode_mixer_in(const float* x, const void* norm_w, const void* w3, void* v0,
                       void* a_out, void* b_hist, const int64_t* t_buf, int max_len, int batch,
                       int d, void* stream);

/* Tree block, gate readout + level recurrence for one position; replaces
 * step_gates_kernel + step_scan_kernel (fused_step.py:26-88, launched at
 * decoding.py:477-486).  Gate weights Wi/Wf/Wr bf16 (L, H, gh), biases fp32
 * (L, H).  ig/fg: fp32 scratch (batch, L, H); counters: int scratch (H),
 * zero before the first call and left zero after each call.  Writes
 * rg_hist[:, t], ring slots of every level at t, and y (batch, d) bf16. */
DH_API int dh_decode_tree_step(const void* a_in, const void* b_hist, const void* wi, const void* wf,
                        const void* wr, const float* bi, const float* bf, const float* br,
                        const int64_t* t_buf, float* ig, float* fg, void* rg_hist,
                        const void* v0, void* v_ring, void* y, int* counters, int batch,
                        int max_len, int L, int H, int hd, int gh, void* stream);

/* x += y . W^T (W: d_out x k, bf16; y bf16 (batch, k)): linear_out and
 * linear_down with the residual add (decoding.py:487-488, 434-435). */
DH_API int dh_decode_linear_residual(const void* y, const void* w, float* x, int batch, int k,
                              int d_out, void* stream);

/* FFN input side: h = RMSNorm(x; norm_w); u = silu(h . Wg^T) * (h . Wu^T),
 * bf16 (batch, ff) (modeling_dispatcher.py:196-197). */
DH_API int dh_decode_ffn_in(const float* x, const void* norm_w, const void* w_gate, const void* w_up,
                     void* u, int batch, int d, int ff, void* stream);

/* Attention block input side (decoding.py:414-426): h = RMSNorm(x);
 * q,k,v = h . [Wq;Wk;Wv]^T; RoPE at position t on q and k (pairs 2j,2j+1,
 * fp32 tables cos/sin (max_len, hd/2)); q -> bf16 (batch, d);
 * k, v -> k_cache / v_cache at t. */
DH_API int dh_decode_attn_in(const float* x, const void* norm_w, const void* wqkv, const float* rope_cos,
                      const float* rope_sin, void* q, void* k_cache, void* v_cache,
                      const int64_t* t_buf, int max_len, int batch, int d, int H, void* stream);

/* Sliding-window attention of q at position t over cache positions
 * (t - window, t] (all of [0, t] when window <= 0); softmax in fp32, scale
 * 1/sqrt(hd) (decoding.py:260-264, 427-433).  Split over `nsplit` chunks of
 * the window; part: fp32 scratch (batch, H, nsplit, hd + 2); counters: int
 * scratch (batch * H), zero before the first call and left zero.  Output y
 * bf16 (batch, H*hd). */
DH_API int dh_decode_attn(const void* q, const void* k_cache, const void* v_cache, void* y,
                   const int64_t* t_buf, float* part, int* counters, int nsplit, int batch,
                   int max_len, int H, int hd, int window, void* stream);

/* logits = RMSNorm(x; norm_w) . E^T, bf16 (batch, vocab) (decoding.py:442). */
DH_API int dh_decode_logits(const float* x, const void* norm_w, const void* emb, void* logits,
                     int batch, int d, int vocab, void* stream);

/* t_buf[0] += 1 (decoding.py:443). */
DH_API int dh_decode_advance(int64_t* t_buf, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DISPATCHER_B200_H */
