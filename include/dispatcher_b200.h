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

/* Poll limit of the bounded device-side waits that report DH_ERR_TIMEOUT
 * (TMA and MMA pipeline waits of the GEMM and gate kernels, the cross-CTA
 * waits of the persistent decode step), read at each launch; polls < 0
 * restores the default (2^26 polls of mbarrier.try_wait, far beyond any
 * legitimate stall), 0 makes every such wait give up at once.  A kernel
 * whose wait gives up skips its later waits, issues no further copies or
 * MMAs, drains what it issued, and returns with *status set: the output is
 * invalid but the context stays usable.  Process-wide; meant for tests of
 * the failure path.  The reference has no counterpart (its Triton kernels
 * have no device-side waits). */
DH_API int dh_set_wait_limit(long long polls);

/* ---------------------------------------------------------------- decode */

/* x[b,:] = fp32(E[tokens[b],:]).  Replaces the embedding lookup of the
 * captured step (decoding.py:438).  Out-of-range ids are clamped and
 * reported by a nonzero *status (nullable). */
DH_API int dh_decode_embed(const int64_t* tokens, const void* emb, float* x, int batch, int d,
                    int vocab, int* status, void* stream);

/* Tree block, mixer input side (decoding.py:473-476): h = RMSNorm(x; norm_w);
 * [v0 | A | B] = h . W3^T with W3 = [W_in; W1x; W1s] (3d x d, bf16);
 * v0, A -> bf16 (batch, d); B -> B_hist[:, t, :].
 * This and the other GEMV entry points below (linear_residual, ffn_in,
 * attn_in, logits) run on the tensor cores with the weights streamed by
 * bulk copies whenever K is a multiple of 32 and the input is 16-byte
 * aligned; *status (nullable) receives DH_ERR_TIMEOUT if one of their
 * bounded pipeline waits gives up. */
DH_API int dh_decode_mixer_in(const float* x, const void* norm_w, const void* w3, void* v0,
                       void* a_out, void* b_hist, const int64_t* t_buf, int max_len, int batch,
                       int d, int* status, void* stream);

/* Tree block, gate readout + level recurrence for one position; replaces
 * step_gates_kernel + step_scan_kernel (fused_step.py:26-88, launched at
 * decoding.py:477-486).  Gate weights Wi/Wf/Wr bf16 (L, H, gh), biases fp32
 * (L, H).  ig/fg: fp32 scratch (batch, L, H); counters: int scratch (H),
 * zero before the first call and left zero after each call.  Writes
 * rg_hist[:, t], ring slots of every level at t, and y (batch, d) bf16.
 * doc_hist (nullable): int (batch, max_len) document id per position; level l
 * is then also masked where doc(t - 2^l) != doc(t), the parallel forward's
 * doc-reset mask (modeling_dispatcher.py:311-323), so prompts may hold
 * several documents (the reference decoder refuses them, decoding.py:89-98). */
DH_API int dh_decode_tree_step(const void* a_in, const void* b_hist, const void* wi, const void* wf,
                        const void* wr, const float* bi, const float* bf, const float* br,
                        const int64_t* t_buf, float* ig, float* fg, void* rg_hist,
                        const void* v0, void* v_ring, void* y, int* counters,
                        const int* doc_hist, int batch, int max_len, int L, int H, int hd, int gh,
                        void* stream);

/* The same tree-block step for lockstep batches (the launch for 3..16 rows;
 * also replaces step_gates_kernel + step_scan_kernel, fused_step.py:26-88,
 * decoding.py:477-486): the gate readouts of one level, all heads and gates
 * at once, run on the tensor cores with relu^2(A + B_hist[t - 2^l]) rounded
 * to bf16 as the mma operand, then one thread per channel runs the level
 * recurrence.  w_gates: bf16 (L * np, gh), row l*np + g*H + h = W_g[l, h]
 * (g = admit, forget, transmit; rows 3H..np-1 zero; np a multiple of 16,
 * at most 48); pre: fp32 scratch (batch, L, np), zero before the first
 * call and left zero after each call.  gh a multiple of 32, hd <= 64.
 * Writes what dh_decode_tree_step writes. */
DH_API int dh_decode_tree_step_tc(const void* a_in, const void* b_hist, const void* w_gates,
                                  int np, const float* bi, const float* bf, const float* br,
                                  const int64_t* t_buf, float* pre, void* rg_hist,
                                  const void* v0, void* v_ring, void* y, const int* doc_hist,
                                  int batch, int max_len, int L, int H, int hd, int gh,
                                  void* stream);

/* Tree block input side with the gate readouts folded in (1..8 rows; the
 * work of dh_decode_mixer_in plus the readout half of dh_decode_tree_step,
 * fused_step.py:26-59): the W3 GEMV as dh_decode_mixer_in, and each 16
 * columns of A it produces add their share of every level's admit / forget /
 * transmit readouts, sum_k W_g[l, h, k] relu(A[b, k] + m B_hist[b, t - 2^l, k])^2
 * (m: the level mask, with doc_hist (nullable) also the document mask), into
 * pre (fp32 (batch, L * np), zero on entry; dh_decode_tree_recur reads and
 * clears it).  w_gates_t: bf16 (d, L * np), the transpose of the packed
 * gate rows of dh_decode_tree_step_tc (column l*np + g*H + h).  d a multiple
 * of 32 and at most 1024; 16 * L * np * 2 bytes at most 33792. */
DH_API int dh_decode_mixer_in_gates(const float* x, const void* norm_w, const void* w3, void* v0,
                                    void* a_out, void* b_hist, const int64_t* t_buf, int max_len,
                                    int batch, int d, const void* w_gates_t, int np, int L, int H,
                                    float* pre, const int* doc_hist, int* status, void* stream);

/* The level recurrence of a tree block from summed gate pre-activations
 * (fused_step.py:62-88): sigmoid gates with the biases bi/bf/br (L, H) and
 * the level / document mask, rg_hist[:, t], every level's ring slot at t and
 * y (batch, d) bf16; pre (batch, L * np) is read and left zero.  One thread
 * per channel and row, every level's history fetched before the dependency
 * wait.  hd <= 64. */
DH_API int dh_decode_tree_recur(const float* bi, const float* bf, const float* br,
                                const int64_t* t_buf, float* pre, int np, void* rg_hist,
                                const void* v0, void* v_ring, void* y, const int* doc_hist,
                                int batch, int max_len, int L, int H, int hd, void* stream);

/* x += y . W^T (W: d_out x k, bf16; y bf16 (batch, k)): linear_out and
 * linear_down with the residual add (decoding.py:487-488, 434-435).  x_copy
 * (nullable) receives a copy of the updated x (the input of dh_decode_ffn). */
DH_API int dh_decode_linear_residual(const void* y, const void* w, float* x, float* x_copy,
                              int batch, int k, int d_out, int* status, void* stream);

/* Whole SwiGLU feed-forward with the residual add, one launch
 * (modeling_dispatcher.py:196-197, decoding.py:434-435, 488):
 * x += silu(RMSNorm(x_in) . Wg^T) * (RMSNorm(x_in) . Wu^T) . Wd^T, u rounded
 * to bf16.  x_in: fp32 (batch, d), a copy of x (from dh_decode_linear_residual);
 * w_down_t: Wd transposed, bf16 (ff, d); x fp32 (batch, d) receives the down
 * projection through atomic adds (summation order not fixed).  d <= 2048.
 * With d <= 1024 (a multiple of 32), for every batch: the gate/up tiles on
 * the tensor cores, all weights streamed by bulk copies, the down projection
 * folded per CTA before its atomic adds; *status (nullable) receives
 * DH_ERR_TIMEOUT if a bounded wait of that pipeline gives up. */
DH_API int dh_decode_ffn(const float* x_in, const void* norm_w, const void* w_gate, const void* w_up,
                  const void* w_down_t, float* x, int batch, int d, int ff, int* status,
                  void* stream);

/* FFN input side: h = RMSNorm(x; norm_w); u = silu(h . Wg^T) * (h . Wu^T),
 * bf16 (batch, ff) (modeling_dispatcher.py:196-197). */
DH_API int dh_decode_ffn_in(const float* x, const void* norm_w, const void* w_gate, const void* w_up,
                     void* u, int batch, int d, int ff, int* status, void* stream);

/* Attention block input side (decoding.py:414-426): h = RMSNorm(x);
 * q,k,v = h . [Wq;Wk;Wv]^T; RoPE at position t on q and k (pairs 2j,2j+1,
 * fp32 tables cos/sin (max_len, hd/2)); q -> bf16 (batch, d);
 * k, v -> k_cache / v_cache at t. */
DH_API int dh_decode_attn_in(const float* x, const void* norm_w, const void* wqkv, const float* rope_cos,
                      const float* rope_sin, void* q, void* k_cache, void* v_cache,
                      const int64_t* t_buf, int max_len, int batch, int d, int H, int* status,
                      void* stream);

/* Sliding-window attention of q at position t over cache positions
 * (t - window, t] (all of [0, t] when window <= 0); softmax in fp32, scale
 * 1/sqrt(hd) (decoding.py:260-264, 427-433).  Split over `nsplit` chunks of
 * the window; part: fp32 scratch (batch, H, nsplit, hd + 2); counters: int
 * scratch (batch * H), zero before the first call and left zero.  Output y
 * bf16 (batch, H*hd). */
DH_API int dh_decode_attn(const void* q, const void* k_cache, const void* v_cache, void* y,
                   const int64_t* t_buf, float* part, int* counters, int nsplit, int batch,
                   int max_len, int H, int hd, int window, void* stream);

/* dh_decode_attn without caller scratch.  No counterpart in the reference
 * (its decoder allocates torch tensors for everything); added for callers that
 * cannot allocate device memory.  Same arguments and result as dh_decode_attn
 * minus part/counters, which live in the library's own static device storage:
 * batch*H*nsplit*(hd+2) <= 131072 floats and batch*H <= 1024, else DH_ERR_SHAPE.
 * The first call on a device sets that device's scratch up (make it before any
 * stream capture).  One scratch area per device: calls that overlap in time on
 * the same device race and must be serialised by the caller. */
DH_API int dh_decode_attn_noalloc(const void* q, const void* k_cache, const void* v_cache, void* y,
                           const int64_t* t_buf, int nsplit, int batch, int max_len, int H,
                           int hd, int window, void* stream);

/* logits = RMSNorm(x; norm_w) . E^T, bf16 (batch, vocab) (decoding.py:442). */
DH_API int dh_decode_logits(const float* x, const void* norm_w, const void* emb, void* logits,
                     int batch, int d, int vocab, int* status, void* stream);

/* Document tracking for multi-document decoding (no counterpart in the
 * reference decoder, which refuses separators in the prompt): doc_hist[b, t]
 * = doc_hist[b, t-1] + (last_tok[b] == eot) (0 at t = 0), then last_tok[b] =
 * tokens[b]; t read from t_buf.  Launch before the step's tree layers. */
DH_API int dh_decode_doc_step(const int64_t* tokens, const int64_t* t_buf, int* doc_hist,
                       int64_t* last_tok, int64_t eot, int batch, int max_len, void* stream);

/* Greedy choice of the next tokens on the device (fast_generate's argmax,
 * modeling_dispatcher.py:433, without a host round trip): per row b, the
 * first index of the largest of logits[b, :] (bf16 (batch, vocab), torch's
 * tie rule), written to next_tokens[b] (the next step's token buffer) and,
 * when out is not null, to out[b]. */
DH_API int dh_decode_argmax(const void* logits, int64_t* next_tokens, int64_t* out, int batch,
                            int vocab, void* stream);

/* Sampling of the next tokens on the device (fast_generate with do_sample,
 * top_k and temperature, modeling_dispatcher.py:426-432, without a host round
 * trip): per row b, a draw from softmax(logits[b] / max(T, 1e-6)) restricted
 * to the logits >= the top_k-th largest (ties at it kept, as the reference's
 * mask), taken as the Gumbel-max over those candidates with uniforms from a
 * counter-based hash of (seed, the position in *t_buf, b, index).  Same
 * distribution as the reference's multinomial; the draws differ.  Writes
 * next_tokens[b] and, when out is not null, out[b]. */
DH_API int dh_decode_sample_top_k(const void* logits, int64_t* next_tokens, int64_t* out, int batch,
                                  int vocab, int top_k, float temperature, unsigned long long seed,
                                  const int64_t* t_buf, void* stream);

/* t_buf[0] += 1 (decoding.py:443). */
DH_API int dh_decode_advance(int64_t* t_buf, void* stream);

/* --------------------------------------------------------------- prefill */

/* C = A . W^T on the tensor cores (tcgen05, TMA, fp32 accumulation): the
 * dense projections of the parallel forward (nn.Linear calls at
 * modeling_dispatcher.py:70-74, 122-123, 171-173, 185, 197, 351).
 * A: M x K bf16 (row stride lda), W: N x K bf16 (row stride ldw), K % 64 == 0.
 * epilogue 0: C = A W^T (bf16, row stride ldc)
 *          1: C = R + A W^T (R bf16, row stride ldr; R may equal C)
 *          2: SwiGLU: W holds gate/up rows interleaved in blocks of 128
 *             (rows [256j, 256j+128) = gate features [128j, 128j+128),
 *             the next 128 = the matching up features); C (M x N/2) =
 *             silu(A Wg^T) * (A Wu^T)  (modeling_dispatcher.py:196-197).
 * status (nullable): set to DH_ERR_TIMEOUT if a bounded pipeline wait gave up. */
DH_API int dh_gemm_bf16(const void* A, int lda, const void* W, int ldw, void* C, int ldc,
                        const void* R, int ldr, int M, int N, int K, int epilogue, int* status,
                        void* stream);

/* Tree mask (modeling_dispatcher.py:282-297, 311-323): mask[b,t,l] = 1 iff
 * 2^l < T, t >= 2^l and (no doc reset, or t and t-2^l lie in the same
 * document, doc = count of `eot` tokens strictly before the position).
 * ids int64 (batch, T); mask uint8 (batch, T, L). */
DH_API int dh_tree_mask(const int64_t* ids, int batch, int T, int L, int64_t eot, int doc_reset,
                        uint8_t* mask, void* stream);

/* Mixer gates for the parallel forward, on the tensor cores; replaces the
 * gate pipeline of fused_gates.py:38-93 / modeling_dispatcher.py:100-114.
 * a, bsrc: A = W1x.x and B = W1s.x, bf16 rows (batch*T, gh), row strides
 * lda/ldb (views into one projection output are fine).  wg: bf16
 * (L*NP, gh), level l rows [l*NP + g*H + h] = gate g (admit, forget,
 * transmit) of head h, rows 3H..NP-1 zero (NP % 16 == 0, NP <= 64).
 * bias fp32 (L, NP) in the same order.  mask: uint8 (batch, T, L) from
 * dh_tree_mask, or NULL for the wrap mask alone.  Levels 0..n_lv-1 go to
 * gates bf16 (batch, H, L, T, 4): per position (admit*m, forget*m + 1-m,
 * transmit, 0), the layout dh_level_scan reads.  When
 * rg_hist is not NULL the transmit gates of all L levels are also written
 * to rg_hist bf16 (batch, rg_T, L, H) (decoder cache, decoding.py:164-174). */
DH_API int dh_mixer_gates(const void* a, int lda, const void* bsrc, int ldb, const void* wg,
                          const float* bias, const uint8_t* mask, int batch, int T, int H, int L,
                          int NP, int gh, int n_lv, void* gates, void* rg_hist, int rg_T,
                          int* status, void* stream);

/* The reference custom op dispatcher::gate_preacts_fwd (fused_gates.py:
 * 186-214, 307-314): pre_i/pre_f/pre_r bf16 (batch, T, n_lv, H) =
 * W_x[l] . relu(A + m*roll(B, 2^l))^2 + b_x, no sigmoid.  Weights and bias
 * packed as for dh_mixer_gates; mask uint8 (batch, T, mask_L) or NULL. */
DH_API int dh_gate_preacts_fwd(const void* a, int lda, const void* bsrc, int ldb, const void* wg,
                               const float* bias, const uint8_t* mask, int mask_L, int batch,
                               int T, int H, int L, int NP, int gh, int n_lv, void* pre_i,
                               void* pre_f, void* pre_r, int* status, void* stream);

/* Backward of dh_gate_preacts_fwd: the reference custom op
 * dispatcher::gate_preacts_bwd (fused_gates.py:96-173, 225-263).  Given
 * dpi/dpf/dpr bf16 (batch, T, n_lv, H), adds into caller-zeroed fp32 outputs
 *   dA, dB (batch, T, gh):  dx = 2 relu(x) (dP . W_l), x = A + m*B(t-2^l);
 *                           dA(t) += dx, dB(t - 2^l) += m dx
 *   dWi/dWf/dWr (n_lv, H, gh) += dP^T . relu(x)^2;  dbi/dbf/dbr (n_lv, H) += sum_t dP
 * (dA is written, not accumulated).  a, bsrc bf16 (batch, T, gh) with row
 * strides lda, ldb; wt bf16 (n_lv*gh, 64): per level W^T with the 3H gate
 * rows (i | f | r) as columns, zero padded; mask uint8 (batch, T, mask_L) or
 * NULL (the wrap mask is always applied).  gh % 64 == 0, 3H <= 48,
 * n_lv <= 16; dpi/dpf/dpr, dA, dB and dW* 16-byte aligned (DH_ERR_ARG
 * otherwise).  status (nullable) is set to DH_ERR_TIMEOUT if a bounded
 * pipeline wait gave up. */
DH_API int dh_gate_preacts_bwd(const void* a, int lda, const void* bsrc, int ldb, const void* wt,
                               const uint8_t* mask, int mask_L, int batch, int T, int H,
                               int n_lv, int gh, const void* dpi, const void* dpf,
                               const void* dpr, float* dA, float* dB, float* dWi, float* dWf,
                               float* dWr, float* dbi, float* dbf, float* dbr, int* status,
                               void* stream);

/* Dyadic level sweep (modeling_dispatcher.py:116-120): for l < n_lv,
 * V(t) <- f_l(t) V(t) + a_l(t) msg(t-2^l), msg = r_l V, in bf16 with the
 * reference's rounding points.  v0 bf16 (batch*T, hd*H)
 * with row stride ld_v0 (heads are contiguous 64-channel groups, the
 * reference's transpose at :70-71); gates from dh_mixer_gates; out bf16
 * with row stride ld_out.  ring (nullable): decoder V_ring (batch, 2^(L+1)-2,
 * H*hd) filled with the last 2^(j+1) positions of each level j
 * (decoding.py:68-76, 154, 179-183).  T <= 4096. */
DH_API int dh_level_scan(const void* v0, int ld_v0, const void* gates, void* out, int ld_out,
                         int batch, int T, int H, int hd, int L, int n_lv, void* ring,
                         void* stream);

/* y = RMSNorm(x) * w over rows of width D, bf16 in/out, fp32 math with the
 * fp32 machine epsilon (torch.nn.RMSNorm, eps=None). */
DH_API int dh_rmsnorm_bf16(const void* x, int ldx, const void* w, void* y, int ldy, int M, int D,
                           void* stream);

/* x[m,:] = E[ids[m],:] (bf16).  Out-of-range ids are clamped and flagged in
 * *status (nullable). */
DH_API int dh_embed_bf16(const int64_t* ids, const void* emb, void* x, int M, int D, int V,
                         int* status, void* stream);

/* In-place RoPE on the q and k thirds of a (M, ld) qkv projection, position
 * m % T, pairs (2j, 2j+1), fp32 tables (max_len, hd/2)
 * (modeling_dispatcher.py:144-166). */
DH_API int dh_rope_qk(void* p, int ld, int M, int T, int d, int hd, const float* rope_cos,
                      const float* rope_sin, void* stream);

/* dst[b, t, 0:n] = src[b*T + t, 0:n] (bf16): fills decoder caches (B_hist,
 * k, v) from prefill activations. */
DH_API int dh_copy_rows(const void* src, int ld_src, void* dst, int ld_dst,
                        long long batch_stride_dst, int batch, int T, int n, void* stream);

/* Sliding-window causal attention over a (batch*T, ld) qkv projection with
 * q, k already rotated: keys s with t - window < s <= t (all s <= t when
 * window <= 0 or window >= T), scale 1/sqrt(hd), hd = 64; out bf16
 * (batch*T, ldo), ldo % 8 == 0 (modeling_dispatcher.py:168-185).  Runs on
 * the 5th-gen tensor cores: S = Q K^T and O += P V with tcgen05.mma
 * (accumulators and P in tensor memory), online softmax in fp32 over blocks
 * of 128 keys.  status (nullable) is set to DH_ERR_TIMEOUT if a bounded
 * pipeline wait gave up. */
DH_API int dh_window_attn_prefill_tc(const void* qkv, int ld, void* out, int ldo, int batch,
                                     int T, int H, int hd, int window, int* status,
                                     void* stream);

/* ------------------------------------------------- persistent decode step */

/* Per-layer weights and caches of the whole-step decode kernel.  Weights
 * are bf16 in packed forms built once by the host; every matrix below is
 * stored row-major with the 16-byte chunks of row r XOR-permuted by (r & 7)
 * (chunk c of row r at position c ^ (r & 7)), r counted from the first row
 * of the matrix (of each 16-row tile for w_gates and w_out of a tree block):
 *   w_in3   tree: [W_in; W1x; W1s] (3d x d); attention: [Wq; Wk; Wv]
 *   w_gates tree: (H, 3, 16, gh): per head, three 16-row tiles (admit,
 *           forget, transmit), row l = that readout of level l, rows >= L zero
 *   b_gates tree: (H, L, 3) fp32 (not permuted)
 *   w_out   tree: (H, d, hd): head h's columns of W_out, row n = W_out[n, h*hd:];
 *           attention: W_out (d x d)
 *   w_gu    (2 ff, d): gate row j at 2j, up row j at 2j + 1
 *   w_down  (ff, d): W_down transposed (row j = column j of W_down) */
typedef struct {
  int kind; /* 0 tree block, 1 attention block */
  const void* norm1;
  const void* norm2;
  const void* w_in3;
  const void* w_gates;
  const float* b_gates;
  const void* w_out;
  const void* w_gu;
  const void* w_down;
  void* b_hist;  /* tree caches (decoding.py:50-66 layouts) */
  void* rg_hist;
  void* v_ring;
  void* k_cache; /* attention caches (decoding.py:79-86) */
  void* v_cache;
} dh_layer_params;

/* uint64 words of the step kernel's hand-off counters (`barrier`) */
#define DH_STEP_SYNC_WORDS 4096

typedef struct {
  int n_layers, batch, d, H, hd, L, ff, vocab, max_len, window, nsplit;
  const int64_t* tokens;  /* (batch) next tokens */
  int64_t* t_buf;         /* position, advanced by the kernel */
  const void* emb;        /* (vocab, d): the embedding rows */
  const void* lm_head;    /* (vocab, d): the (tied) output head, rows permuted as above */
  const void* norm_out;
  const float* rope_cos;  /* (max_len, hd/2) fp32 */
  const float* rope_sin;
  const dh_layer_params* layers; /* device array of n_layers */
  void* logits;           /* bf16 (batch, vocab) */
  /* caller-provided device memory:
   * x, x_in fp32 (batch, d): the residual stream and the FFN's copy of it;
   * a, v0, y, q bf16 (batch, d); part fp32 (batch, H, nsplit, hd + 2);
   * counters int (H + batch*H), zero; barrier uint64 [DH_STEP_SYNC_WORDS],
   * zero before the first step (word 0 counts steps, the others are the
   * phases' hand-off counters); status int [1] */
  float* x;
  float* x_in;
  void* a;
  void* v0;
  void* y;
  void* q;
  float* part;
  int* counters;
  unsigned long long* barrier;
  int* status;
  /* nullable: when set, thread 0 of CTA c writes the global timer (ns) at
   * trace[c * DH_STEP_TRACE_WORDS + (layer * 5 + phase) * 4 + k] for k =
   * 0 phase entry, 1 after its hand-off wait, 2 after its input staging,
   * 3 before its arrival (phase: 0 projections, 1 gates / attention,
   * 2 attention out-projection, 3 FFN; at layer n_layers: phase 0 the
   * logits, phase 1 k = 0, 1 the CTA's start and end) */
  unsigned long long* trace;
} dh_step_params;

#define DH_STEP_TRACE_WORDS 512

/* One whole lockstep decode step (embedding, every block, logits, t += 1)
 * as ONE persistent cooperative kernel, one CTA per SM: the last 2H CTAs
 * run each head's gate readouts, level recurrence and share of the output
 * projection, the others the projections and the FFN, every contraction on
 * the tensor cores (mma.sync m16n8k16); each CTA streams its
 * weight slices by bulk copies into shared memory ahead of the phase
 * hand-offs (monotonic per-phase counters, bounded waits: a timeout sets
 * *status = DH_ERR_TIMEOUT and the kernel still runs to completion).
 * Replaces the captured per-token graph of decoding.py:437-443 with the
 * fused tree step of decoding.py:457-488 (fused_step.py:26-88) and the
 * attention step of decoding.py:411-435.  batch <= 2, hd == 64, d a multiple
 * of 128 up to 1024, L * (2 d + 16) <= 32768.
 * `params` is a host pointer; its `layers` array must already be in device
 * memory. */
DH_API int dh_decode_step(const dh_step_params* params, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DISPATCHER_B200_H */
