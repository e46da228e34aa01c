// Whole decode step as ONE persistent cooperative kernel (one CTA per SM).
//
// Roles.  The last H CTAs are "head" CTAs (one per attention head of the
// mixer); the others are "GEMV" CTAs.  A tree block is three dependent
// phases:
//   A  (GEMV CTAs)  h = RMSNorm(x); [v0 | A | B_hist[t]] = W3 h
//   B  (head CTAs)  head h: the gate readouts of all levels
//                   (relu^2(A + B_hist[t - 2^l]) . W_l), the level recurrence
//                   over the ring buffers, and the head's share of the output
//                   projection, added into the residual with vector atomics
//   C  (GEMV CTAs)  h2 = RMSNorm(x); u = silu(Wg h2) * (Wu h2) for this CTA's
//                   slice of the FFN width; x += Wd[:, slice] u (vector atomics)
// An attention block is A (q, k, v with RoPE, cache write), B (window
// attention split over the GEMV CTAs, last-arriver combine), O (output
// projection, rows owned) and C.  The step ends with the logits on all CTAs.
// This follows the reference's fused step (decoding.py:457-488 with
// fused_step.py:26-88) and attention step (decoding.py:411-435).
//
// Weights never depend on activations, so each CTA's producer lane streams
// its slices of every phase of the step, in consumption order, by bulk async
// copies (cp.async.bulk) into a ring of shared-memory slots that runs ahead of
// the phase waits; history rows the head CTAs need (B_hist at t - 2^l)
// travel in the same stream, and ring slots, transmit gates at the source
// positions and the attention window's keys and values (all written by
// earlier steps) are loaded before each wait.  After a wait a phase reads
// only the small activation vector and computes from shared memory.
//
// Hand-off: a phase's CTAs add 1 to its own monotonically increasing 64-bit
// counter with release semantics after their writes; waiters spin on it with
// acquire loads up to a bounded number of polls.  The residual stream lives in
// two fp32 buffers: xb accumulates (C adds into it, the next A reads it), xa
// is the input of C (A copies xb into it, B or O adds into both).
//
// Failure path: every wait is bounded.  A wait that gives up sets *status to
// DH_ERR_TIMEOUT and an abort flag in shared memory; from then on the CTA
// skips its waits (computing garbage but always arriving, so the counters
// stay consistent), the producer issues no further copies and, before the
// CTA exits, waits (with a fixed bound) for the copies it issued.
#include <math.h>

#include "common.cuh"

namespace dh {
namespace {

constexpr int kWarps = 8;                    // consumer warps
constexpr int kCons = kWarps * 32;           // consumer threads
constexpr int kThreads = kCons + 128;        // + the producer warpgroup (one lane issues the copies)
// register split after launch (168 per thread at launch: 384 x 168 = 64512):
// producer warpgroup 128 x 56 + consumers 256 x 224 = 64512
constexpr int kProdRegs = 56;
constexpr int kConsRegs = 224;
static_assert(128 * kProdRegs + kCons * kConsRegs <= kThreads * 168, "register split exceeds the launch");
constexpr int kSlotBytes = 32 * 1024;
// ring depth: 5 slots up to 2 lockstep rows, 4 from 4 rows (their staging needs the room)
template <int MAXB>
constexpr int slots_for() { return MAXB >= 4 ? 4 : 5; }
constexpr int kKvPos = 128;                  // window positions staged per attention item
constexpr int kHeadParts = 2;                // head CTAs per head (each takes half the out-projection rows)
constexpr int kLgMax = 4;                    // levels per gate chunk
constexpr int kLmax = 16;
constexpr int kMaxUpc = 32;                  // FFN elements per GEMV CTA
constexpr float kEps = 1.1920928955078125e-07f;  // torch RMSNorm eps=None in fp32
constexpr uint32_t kDrainLimit = 1u << 20;
constexpr int kSyncStride = 32;              // uint64 words between two phase counters
constexpr int kMaxLayers = DH_STEP_SYNC_WORDS / kSyncStride / 5 - 1;  // hand-off counters available

enum { PH_A = 0, PH_B = 1, PH_O = 2, PH_C = 3, PH_N = 4 };

__device__ __forceinline__ void split_range(int n, int parts, int i, int& a, int& b) {
  a = (int)((long long)n * i / parts);
  b = (int)((long long)n * (i + 1) / parts);
}

__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kCons) : "memory"); }

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_u64(unsigned long long* p) {
  asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(p) : "memory");
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// After this, lane l holds the warp-wide sum of v[l % NV] (NV a power of two <= 32).
template <int NV>
__device__ __forceinline__ float transpose_reduce(float (&v)[NV]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int n = NV; n > 1; n >>= 1) {
    const int o = n >> 1;
    const bool upper = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = upper ? v[i] : v[i + n / 2];
      const float keep = upper ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  float r = v[0];
#pragma unroll
  for (int o = NV; o < 32; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
  return r;
}

// ------------------------------------------------------------------ the plan
// A segment is a run of equal units of one weight matrix (or of history rows)
// that this CTA streams for one phase; chunks are whole units, <= one slot.
enum { SEG_ROWS = 0, SEG_GATES = 1 };
struct Seg {
  const uint8_t* base;
  uint32_t unit_bytes;  // SEG_GATES: bytes of one level's weights (3 gh bf16)
  int units;
  int kind;
  size_t limit;         // bytes readable from base (the last unit may be short)
};

struct Ctx {
  const dh_step_params& p;
  int G, cta, NG, head;  // head >= 0 on head CTAs
  int hpart;             // which half of the head's out-projection rows
  int B, d, gh, L, H, hd, ff;
  long long t;
  unsigned long long gen;
  uint32_t wait_limit;
  int nsplit;            // attention splits per (row, head)
  int lg;                // levels per gate chunk
  int nslots;            // ring slots
  // shared memory
  uint8_t* slots;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort;
  __nv_bfloat16* xs;     // staged activation rows [MAXB][1024]
  float* red;            // reductions
  float* misc;           // small per-phase arrays
  __nv_bfloat16* kv;     // [2][kKvPos][hd]
  int consumed;          // chunks consumed (same in every consumer thread)
  struct Prod* prod;     // the weight stream (shared memory; the producer lane)
  const dh_layer_params* lay;  // the layer table, copied into shared memory
};

// The weight stream's state, in shared memory, used by the producer lane: a
// copy of the CTA's geometry and the cursor of the next chunk.
struct Prod {
  const dh_step_params* pp;
  const dh_layer_params* lay;  // shared-memory copy of the layer table
  const void* emb;
  int vocab, max_len, n_layers;
  int G, cta, NG, head, hpart, B, d, gh, L, H, hd, ff, lg, nslots;
  long long t;
  uint32_t wait_limit;
  uint8_t* slots;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort;
  int cli, cph, csi, cu;  // next chunk: layer, phase, segment, unit
  Seg cseg;
  int cvalid;             // a chunk is left to issue
  int pslot;              // ring slot of the next chunk
  uint32_t peph;          // parity of that slot's empty barrier to wait for
  long issued;            // chunks issued so far
};

// the few step parameters the plan needs, for both the consumers' context
// and the issuer's shared-memory copy
__device__ __forceinline__ int vocab_of(const Ctx& c) { return c.p.vocab; }
__device__ __forceinline__ int vocab_of(const Prod& c) { return c.vocab; }
__device__ __forceinline__ const void* emb_of(const Ctx& c) { return c.p.emb; }
__device__ __forceinline__ const void* emb_of(const Prod& c) { return c.emb; }

template <class C>
__device__ __forceinline__ const dh_layer_params& layer(const C& c, int li) { return c.lay[li]; }

// optional timeline: global timer of (layer, phase, event k) by thread 0
__device__ __forceinline__ void stamp(const Ctx& c, int li, int ph, int k) {
  if (c.p.trace && threadIdx.x == 0) {
    unsigned long long ns;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ns));
    c.p.trace[(size_t)c.cta * DH_STEP_TRACE_WORDS + (li * 5 + ph) * 4 + k] = ns;
  }
}

// number of segments of (layer li, phase ph) for this CTA, and segment si
template <class C>
__device__ int seg_count(const C& c, int li, int ph) {
  if (ph == PH_N) return 1;
  const bool tree = layer(c, li).kind == 0;
  if (c.head >= 0) return (tree && ph == PH_B) ? 2 : 0;
  if (ph == PH_A || ph == PH_O) return (ph == PH_O && tree) ? 0 : 1;
  if (ph == PH_C) return 2;
  return 0;
}

template <class C>
__device__ Seg get_seg(const C& c, int li, int ph, int si) {
  Seg s{nullptr, 1, 0, SEG_ROWS, 0};
  const int d = c.d;
  if (ph == PH_N) {  // lm_head row pairs, split over every CTA
    int u0, u1;
    const int units = (vocab_of(c) + 1) / 2;
    split_range(units, c.G, c.cta, u0, u1);
    s.base = static_cast<const uint8_t*>(emb_of(c)) + (size_t)u0 * 4 * d;
    s.unit_bytes = 4 * d;
    s.units = u1 - u0;
    s.limit = (size_t)vocab_of(c) * d * 2 - (size_t)u0 * 4 * d;
    return s;
  }
  const dh_layer_params& lp = layer(c, li);
  if (c.head >= 0) {  // tree block B: gates (+ history rows), then the out-projection block
    if (si == 0) {
      s.base = static_cast<const uint8_t*>(lp.w_gates) + (size_t)c.head * c.L * 3 * c.gh * 2;
      s.unit_bytes = 3 * c.gh * 2;
      s.units = c.L;
      s.kind = SEG_GATES;
    } else {  // this CTA's half of the output rows, head h's columns
      s.base = static_cast<const uint8_t*>(lp.w_out) +
               ((size_t)c.head * d + (size_t)c.hpart * (d / kHeadParts)) * c.hd * 2;
      s.unit_bytes = 32 * c.hd * 2;  // 32 output rows
      s.units = d / kHeadParts / 32;
    }
    s.limit = (size_t)s.units * s.unit_bytes;
    return s;
  }
  const int gi = c.cta;
  int u0, u1;
  if (ph == PH_A || ph == PH_O) {  // row pairs of W3 / Wqkv / W_out
    const int units = ph == PH_A ? 3 * d / 2 : d / 2;
    split_range(units, c.NG, gi, u0, u1);
    s.base = static_cast<const uint8_t*>(ph == PH_A ? lp.w_in3 : lp.w_out) + (size_t)u0 * 4 * d;
    s.unit_bytes = 4 * d;
  } else {  // PH_C: (gate, up) row pairs, then rows of Wd^T, for the same FFN slice
    split_range(c.ff, c.NG, gi, u0, u1);
    if (si == 0) {
      s.base = static_cast<const uint8_t*>(lp.w_gu) + (size_t)u0 * 4 * d;
      s.unit_bytes = 4 * d;
    } else {
      s.base = static_cast<const uint8_t*>(lp.w_down) + (size_t)u0 * 2 * d;
      s.unit_bytes = 2 * d;
    }
  }
  s.units = u1 - u0;
  s.limit = (size_t)s.units * s.unit_bytes;
  return s;
}

template <class C>
__device__ __forceinline__ int units_per_chunk(const C& c, const Seg& s) {
  if (s.kind == SEG_GATES) return c.lg;
  const int n = kSlotBytes / (int)s.unit_bytes;
  return n < 1 ? 1 : n;
}

// bytes of a gate chunk: levels [l0, l1) of weights, then the history rows
// B_hist[b, t - 2^l] of those levels for every lockstep row
template <class C>
__device__ __forceinline__ uint32_t gate_chunk_bytes(const C& c, int l0, int l1) {
  return (uint32_t)(l1 - l0) * 3 * c.gh * 2 + (uint32_t)(l1 - l0) * c.B * c.gh * 2;
}

// ------------------------------------------------------------------ the weight stream
// The producer lane issues the CTA's chunks in plan order, each as soon as
// every consumer warp released the slot: for every layer the phases A, B, O,
// C in order, then the logits; in each phase this CTA's segments.
// move the cursor to the first non-empty segment at or after (li, ph, si)
__device__ __forceinline__ void cursor_seek(Prod* pr, int li, int ph, int si) {
  const int nl = pr->n_layers;
  for (; li <= nl; ++li, ph = 0, si = 0) {
    for (; ph < 5; ++ph, si = 0) {
      if ((li == nl) != (ph == PH_N)) continue;
      const int ns = seg_count(*pr, li, ph);
      for (; si < ns; ++si) {
        const Seg sg = get_seg(*pr, li, ph, si);
        if (sg.units > 0) {
          pr->cli = li;
          pr->cph = ph;
          pr->csi = si;
          pr->cu = 0;
          pr->cseg = sg;
          pr->cvalid = 1;
          return;
        }
      }
    }
  }
  pr->cvalid = 0;
}

// issue the chunk under the cursor into the next slot and advance
__device__ __forceinline__ void issue_chunk(Prod* pr) {
  const Seg s = pr->cseg;
  const int upc = units_per_chunk(*pr, s);
  const int u = pr->cu, n = min(upc, s.units - u);
  const int slot = pr->pslot;
  uint8_t* dst = pr->slots + (size_t)slot * kSlotBytes;
  uint64_t* bar = &pr->full[slot];
  if (s.kind == SEG_GATES) {
    const dh_layer_params& lp = layer(*pr, pr->cli);
    const uint32_t wbytes = (uint32_t)n * s.unit_bytes;
    const int B = pr->B, gh = pr->gh;
    const long long t = pr->t;
    uint32_t total = wbytes;
    for (int l = u; l < u + n; ++l)
      if (t - (1ll << l) >= 0) total += (uint32_t)B * gh * 2;
    mbar_arrive_expect_tx(bar, total);
    bulk_g2s(dst, s.base + (size_t)u * s.unit_bytes, wbytes, bar);
    const __nv_bfloat16* bh = static_cast<const __nv_bfloat16*>(lp.b_hist);
    for (int l = u; l < u + n; ++l) {
      const long long src = t - (1ll << l);
      if (src < 0) continue;
      for (int b = 0; b < B; ++b)
        bulk_g2s(dst + wbytes + ((size_t)(l - u) * B + b) * gh * 2,
                 bh + ((size_t)b * pr->max_len + src) * gh, (uint32_t)gh * 2, bar);
    }
  } else {
    const size_t off = (size_t)u * s.unit_bytes;
    size_t bytes = (size_t)n * s.unit_bytes;
    if (off + bytes > s.limit) bytes = s.limit - off;
    mbar_arrive_expect_tx(bar, (uint32_t)bytes);
    bulk_g2s(dst, s.base + off, (uint32_t)bytes, bar);
  }
  ++pr->issued;
  if (++pr->pslot == pr->nslots) {
    pr->pslot = 0;
    pr->peph ^= 1;
  }
  pr->cu = u + n;
  if (pr->cu >= s.units) cursor_seek(pr, pr->cli, pr->cph, pr->csi + 1);
}

// The producer (one lane of the last warp): walks the plan, waiting (bounded)
// for each slot to be released by every consumer warp before refilling it;
// stops at the first failed wait or when a consumer aborted, and finally waits
// (with a fixed bound) for the copies it issued.
__device__ void producer(Prod* pr, int* status) {
  while (pr->cvalid && !*pr->abort) {
    if (pr->issued >= pr->nslots &&
        !mbar_wait(&pr->empty[pr->pslot], pr->peph ^ 1, status, pr->wait_limit)) {
      *pr->abort = 1;
      break;
    }
    if (*pr->abort) break;
    issue_chunk(pr);
  }
  for (int s = 0; s < pr->nslots; ++s) {
    const long n_s = pr->issued / pr->nslots + (s < pr->issued % pr->nslots ? 1 : 0);
    if (n_s > 0) mbar_wait(&pr->full[s], (uint32_t)((n_s - 1) & 1), nullptr, kDrainLimit);
  }
}

// ------------------------------------------------------------------ consumer helpers
__device__ __forceinline__ const uint8_t* chunk_acquire(Ctx& c) {
  const int slot = c.consumed % c.nslots;
  if (!*c.abort) {
    if (!mbar_wait(&c.full[slot], (uint32_t)((c.consumed / c.nslots) & 1), c.p.status, c.wait_limit))
      *c.abort = 1;
  }
  return c.slots + (size_t)slot * kSlotBytes;
}

__device__ __forceinline__ void chunk_release(Ctx& c) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&c.empty[c.consumed % c.nslots]);
  c.consumed += 1;
}

__device__ __forceinline__ unsigned long long* phase_ctr(const Ctx& c, int li, int ph) {
  return c.p.barrier + (size_t)(1 + li * 5 + ph) * kSyncStride;
}

// all consumer threads: wait until `arrivals` CTAs have finished phase (li, ph)
__device__ __forceinline__ void grid_wait(Ctx& c, int li, int ph, int arrivals) {
  if (threadIdx.x == 0 && !*c.abort) {
    const unsigned long long* ctr = phase_ctr(c, li, ph);
    const unsigned long long target = (c.gen + 1) * (unsigned long long)arrivals;
    // each poll is an L2 round trip (~1 us): 1/32 of the mbarrier poll limit
    // (2^21 polls, about two seconds, at the default)
    const uint32_t limit = c.wait_limit >> 5;
    uint32_t it = 0;
    while (ld_acquire_u64(ctr) < target) {
      if (++it > limit) {
        atomicExch(c.p.status, DH_ERR_TIMEOUT);
        *c.abort = 1;
        break;
      }
    }
  }
  csync();
}

// all consumer threads: this CTA has finished phase (li, ph)
__device__ __forceinline__ void grid_arrive(Ctx& c, int li, int ph) {
  csync();
  if (threadIdx.x == 0) red_release_u64(phase_ctr(c, li, ph));
}

// xs[b][k] = bf16(x[b][k] * rsqrt(mean(x[b]^2) + eps) * w[k]) for every lockstep row;
// x comes from `xf` (fp32, read through L2) or, for the first block, from the
// embedding rows of the step's tokens.  The same loads also write this CTA's
// slice [e0, e1) (float4 units) of x into dst0 / dst1 when they are set.
template <int MAXB>
__device__ void stage_norm(Ctx& c, const float* xf, const __nv_bfloat16* w, float* dst0 = nullptr,
                           float* dst1 = nullptr, int e0 = 0, int e1 = 0) {
  const int B = c.B, d = c.d, d4 = d / 4, n4 = B * d4;
  constexpr int NV = (MAXB * 1024 + kCons * 4 - 1) / (kCons * 4);
  float* ssum = c.red;  // [MAXB]
  if (threadIdx.x < MAXB) ssum[threadIdx.x] = 0.f;
  float4 v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * kCons;
    if (i < n4) {
      const int b = i / d4, k = (i - b * d4) * 4;
      if (xf) {
        v[j] = __ldcg(reinterpret_cast<const float4*>(xf + (size_t)b * d + k));
      } else {
        long long tok = c.p.tokens[b];
        if (tok < 0 || tok >= c.p.vocab) tok = 0;  // reported by the phase that owns the row
        const uint2 e = *reinterpret_cast<const uint2*>(static_cast<const __nv_bfloat16*>(c.p.emb) +
                                                        (size_t)tok * d + k);
        const float2 e01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&e.x));
        const float2 e23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&e.y));
        v[j] = make_float4(e01.x, e01.y, e23.x, e23.y);
      }
    }
  }
  csync();  // ssum cleared
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * kCons;
    float sq = 0.f;
    if (i < n4) {
      sq = v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
      if (i >= e0 && i < e1) {
        const size_t off = (size_t)(i / d4) * d + (i - (i / d4) * d4) * 4;
        if (dst0) *reinterpret_cast<float4*>(dst0 + off) = v[j];
        if (dst1) *reinterpret_cast<float4*>(dst1 + off) = v[j];
      }
    }
    if ((d4 & 31) == 0) {  // a warp's 32 float4 lie in one row: reduce, one atomic
      sq = warp_sum(sq);
      if ((threadIdx.x & 31) == 0 && i < n4) atomicAdd(&ssum[i / d4], sq);
    } else if (i < n4) {
      atomicAdd(&ssum[i / d4], sq);
    }
  }
  csync();
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * kCons;
    if (i < n4) {
      const int b = i / d4, k = (i - b * d4) * 4;
      const float r = rsqrtf(ssum[b] / (float)d + kEps);
      const uint2 wv = *reinterpret_cast<const uint2*>(w + k);
      const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.x));
      const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.y));
      uint2 pk;
      pk.x = pack2(v[j].x * r * w01.x, v[j].y * r * w01.y);
      pk.y = pack2(v[j].z * r * w23.x, v[j].w * r * w23.y);
      *reinterpret_cast<uint2*>(c.xs + (size_t)b * 1024 + k) = pk;
    }
  }
  csync();
}

// xs[b][0:K] = src[b][0:K] (bf16 produced by another CTA)
__device__ void stage_copy(Ctx& c, const __nv_bfloat16* src, int K) {
  const int k8 = K / 8, n = c.B * k8;
  for (int i = threadIdx.x; i < n; i += kCons) {
    const int b = i / k8, k = (i - b * k8) * 8;
    *reinterpret_cast<uint4*>(c.xs + (size_t)b * 1024 + k) =
        __ldcg(reinterpret_cast<const uint4*>(src + (size_t)b * K + k));
  }
  csync();
}

// acc[0..MAXB) += row r0 . xs[b], acc[MAXB..2MAXB) += row r1 . xs[b]  (this lane's k slice)
template <int MAXB>
__device__ __forceinline__ void dot_pair(const __nv_bfloat16* r0, const __nv_bfloat16* r1, int K,
                                         const __nv_bfloat16* xs, int B, float (&acc)[2 * MAXB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 2 * MAXB; ++i) acc[i] = 0.f;
  uint4 wa[4], wb[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {  // K <= 1024: every load of the row pair up front
    const int k = lane * 8 + i * 256;
    if (k < K) {
      wa[i] = *reinterpret_cast<const uint4*>(r0 + k);
      wb[i] = *reinterpret_cast<const uint4*>(r1 + k);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int k = lane * 8 + i * 256;
    if (k >= K) break;
    float fa[8], fb[8];
    unpack8(wa[i], fa);
    unpack8(wb[i], fb);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < B) {
        float fx[8];
        unpack8(*reinterpret_cast<const uint4*>(xs + (size_t)b * 1024 + k), fx);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[b] = fmaf(fa[j], fx[j], acc[b]);
          acc[MAXB + b] = fmaf(fb[j], fx[j], acc[MAXB + b]);
        }
      }
    }
  }
}

// Consume segment `s` (row pairs of a K-wide matrix) against xs; `store(u, b,
// row, v, other, has1)` receives unit u's row `row` for lockstep row b.
template <int MAXB, class Store>
__device__ void gemv_segment(Ctx& c, const Seg& s, int K, int unit0, Store store) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int upc = units_per_chunk(c, s);
  for (int cu = 0; cu < s.units; cu += upc) {
    const int n = min(upc, s.units - cu);
    const uint8_t* chunk = chunk_acquire(c);
    for (int u = warp; u < n; u += kWarps) {
      const size_t off = (size_t)(cu + u) * s.unit_bytes;
      const __nv_bfloat16* r0 = reinterpret_cast<const __nv_bfloat16*>(chunk + (size_t)u * s.unit_bytes);
      const bool has1 = off + s.unit_bytes <= s.limit;
      const __nv_bfloat16* r1 = has1 ? r0 + K : r0;
      float acc[2 * MAXB];
      dot_pair<MAXB>(r0, r1, K, c.xs, c.B, acc);
      const float r = transpose_reduce<2 * MAXB>(acc);
      const float other = __shfl_xor_sync(0xffffffffu, r, MAXB);
      const int b = lane % MAXB, row = (lane / MAXB) & 1;
      if (lane < 2 * MAXB && b < c.B && (row == 0 || has1)) store(unit0 + cu + u, b, row, r, other);
    }
    chunk_release(c);
  }
}

// ------------------------------------------------------------------ phases
template <int MAXB>
__device__ void phase_a(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  const bool tree = lp.kind == 0;
  const int d = c.d, B = c.B;
  stamp(c, li, PH_A, 0);
  if (li > 0) grid_wait(c, li - 1, PH_C, c.NG);
  stamp(c, li, PH_A, 1);
  // the residual: layer 0 starts it (both buffers) from the embedding rows; a
  // tree block copies its accumulated value into x_in (the input of C, which
  // B adds into); each CTA writes its slice, from the loads of the staging
  {
    int e0, e1;
    split_range(B * d / 4, c.NG, c.cta, e0, e1);
    if (li == 0 && threadIdx.x < B && c.cta == 0) {
      const long long tok = c.p.tokens[threadIdx.x];
      if (tok < 0 || tok >= c.p.vocab) atomicExch(c.p.status, DH_ERR_ARG);
    }
    stage_norm<MAXB>(c, li == 0 ? nullptr : c.p.x, static_cast<const __nv_bfloat16*>(lp.norm1),
                     li == 0 ? c.p.x : nullptr, (li == 0 || tree) ? c.p.x_in : nullptr, e0, e1);
  }
  stamp(c, li, PH_A, 2);
  const Seg s = get_seg(c, li, PH_A, 0);
  int u0, u1;
  split_range(3 * d / 2, c.NG, c.cta, u0, u1);
  const long long t = c.t;
  if (tree) {
    __nv_bfloat16* v0 = static_cast<__nv_bfloat16*>(c.p.v0);
    __nv_bfloat16* a = static_cast<__nv_bfloat16*>(c.p.a);
    __nv_bfloat16* bh = static_cast<__nv_bfloat16*>(lp.b_hist);
    const int ml = c.p.max_len;
    gemv_segment<MAXB>(c, s, d, u0, [&](int u, int b, int row, float v, float) {
      const int n = 2 * u + row, seg = n / d, col = n - seg * d;
      if (seg == 0) v0[(size_t)b * d + col] = f2bf(v);
      else if (seg == 1) a[(size_t)b * d + col] = f2bf(v);
      else bh[((size_t)b * ml + t) * d + col] = f2bf(v);
    });
  } else {
    __nv_bfloat16* q = static_cast<__nv_bfloat16*>(c.p.q);
    __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(lp.k_cache);
    __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(lp.v_cache);
    const int ml = c.p.max_len, hd = c.hd;
    const float* cosT = c.p.rope_cos;
    const float* sinT = c.p.rope_sin;
    gemv_segment<MAXB>(c, s, d, u0, [&](int u, int b, int row, float v, float other) {
      const int n = 2 * u + row, seg = n / d, col = n - seg * d;
      float out = v;
      if (seg < 2) {  // rotate the pair (2j, 2j+1) of q and k at position t
        const int j = (col % hd) >> 1;
        const float cs = cosT[t * (hd / 2) + j], sn = sinT[t * (hd / 2) + j];
        const float x1 = row == 0 ? v : other, x2 = row == 0 ? other : v;
        out = row == 0 ? (x1 * cs - x2 * sn) : (x1 * sn + x2 * cs);
      }
      if (seg == 0) q[(size_t)b * d + col] = f2bf(out);
      else if (seg == 1) kc[((size_t)b * ml + t) * d + col] = f2bf(out);
      else vc[((size_t)b * ml + t) * d + col] = f2bf(out);
    });
  }
  stamp(c, li, PH_A, 3);
  grid_arrive(c, li, PH_A);
}

// head CTA: gates of every level, level recurrence, out-projection share
template <int MAXB>
__device__ void phase_b_tree(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  const int B = c.B, L = c.L, H = c.H, hd = c.hd, gh = c.gh, d = c.d, h = c.head;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long t = c.t;
  const int ml = c.p.max_len;
  const int S = (1 << (L + 1)) - 2;
  __nv_bfloat16* ring = static_cast<__nv_bfloat16*>(lp.v_ring);
  __nv_bfloat16* rg = static_cast<__nv_bfloat16*>(lp.rg_hist);
  // small arrays in c.misc
  float* s_f = c.misc;                        // [MAXB][kLmax]
  float* s_c = s_f + MAXB * kLmax;            // [MAXB][kLmax]
  float* s_rg = s_c + MAXB * kLmax;           // [MAXB][kLmax] transmit gate at the source
  float* s_y = s_rg + MAXB * kLmax;           // [MAXB][64]
  uint4* s_v0 = reinterpret_cast<uint4*>(s_y + MAXB * 64);                   // [MAXB][8]
  __nv_bfloat16* s_ring = reinterpret_cast<__nv_bfloat16*>(s_v0 + MAXB * 8);  // [MAXB][kLmax][64]
  stamp(c, li, PH_B, 0);
  // history written by earlier steps: ring slots of the source positions and
  // their transmit gates (one round trip, before the wait)
  for (int i = tid; i < B * L * 8; i += kCons) {
    const int b = i / (L * 8), r = i - b * (L * 8), l = r / 8, g = r - l * 8;
    const long long src = t - (1ll << l);
    uint4 v = make_uint4(0, 0, 0, 0);
    if (src >= 0) {
      const long long slot = ((2ll << l) - 2) + (src & ((2ll << l) - 1));
      v = *reinterpret_cast<const uint4*>(ring + ((size_t)b * S + slot) * d + h * hd + g * 8);
    }
    *reinterpret_cast<uint4*>(s_ring + ((size_t)b * kLmax + l) * 64 + g * 8) = v;
    if (g == 0)
      s_rg[b * kLmax + l] = src >= 0 ? bf2f(rg[(((size_t)b * ml + src) * L + l) * H + h]) : 0.f;
  }
  grid_wait(c, li, PH_A, c.NG);
  stamp(c, li, PH_B, 1);
  // A rows (every column) and this head's v0 slice, one round trip
  {
    const __nv_bfloat16* a = static_cast<const __nv_bfloat16*>(c.p.a);
    const __nv_bfloat16* v0 = static_cast<const __nv_bfloat16*>(c.p.v0);
    const int k8 = gh / 8, n = B * k8;
    for (int i = tid; i < n + B * 8; i += kCons) {
      if (i < n) {
        const int b = i / k8, k = (i - b * k8) * 8;
        *reinterpret_cast<uint4*>(c.xs + (size_t)b * 1024 + k) =
            __ldcg(reinterpret_cast<const uint4*>(a + (size_t)b * gh + k));
      } else {
        const int j = i - n, b = j / 8, g = j - b * 8;
        s_v0[b * 8 + g] = __ldcg(reinterpret_cast<const uint4*>(v0 + (size_t)b * d + h * hd + g * 8));
      }
    }
  }
  csync();
  stamp(c, li, PH_B, 2);
  // gate readouts, chunk by chunk (a chunk holds up to kLgMax levels: their
  // weights, then their history rows): thread tid owns columns [4 tid, 4 tid + 4)
  // of the hidden width; all loads of a chunk are issued before its FMAs and
  // its (level, gate) partial sums leave in one transpose reduction per row
  float* red = c.red;  // [kWarps][MAXB][kLmax * 3]
  const int k = tid * 4;
  const bool kin = k < gh;
  const Seg sg = get_seg(c, li, PH_B, 0);
  for (int l0 = 0; l0 < L; l0 += c.lg) {
    const int nlv = min(L, l0 + c.lg) - l0;
    const uint8_t* chunk = chunk_acquire(c);
    const uint32_t wbytes = (uint32_t)nlv * sg.unit_bytes;
    for (int b = 0; b < B; ++b) {
      const uint2 au = kin ? *reinterpret_cast<const uint2*>(c.xs + (size_t)b * 1024 + k) : make_uint2(0, 0);
      float av[4];
      {
        const float2 a01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&au.x));
        const float2 a23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&au.y));
        av[0] = a01.x; av[1] = a01.y; av[2] = a23.x; av[3] = a23.y;
      }
      uint2 bu[kLgMax];
#pragma unroll
      for (int j = 0; j < kLgMax; ++j) {
        const bool ok = j < nlv && kin && t - (1ll << (l0 + j)) >= 0;
        bu[j] = ok ? *reinterpret_cast<const uint2*>(chunk + wbytes + (((size_t)j * B + b) * gh + k) * 2)
                   : make_uint2(0, 0);
      }
      float acc[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) acc[q] = 0.f;
#pragma unroll
      for (int j = 0; j < kLgMax; ++j) {
        const float2 b01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bu[j].x));
        const float2 b23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&bu[j].y));
        const float bs[4] = {b01.x, b01.y, b23.x, b23.y};
        float hv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = fmaxf(av[e] + bs[e], 0.f);
          hv[e] = x * x;  // relu squared
        }
#pragma unroll
        for (int g = 0; g < 3; ++g) {
          const uint2 wq = (j < nlv && kin)
              ? *reinterpret_cast<const uint2*>(chunk + ((size_t)j * 3 * gh + (size_t)g * gh + k) * 2)
              : make_uint2(0, 0);
          const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wq.x));
          const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wq.y));
          acc[j * 3 + g] = fmaf(w01.x, hv[0], fmaf(w01.y, hv[1], fmaf(w23.x, hv[2], w23.y * hv[3])));
        }
      }
      const float r = transpose_reduce<16>(acc);
      if (lane < nlv * 3) red[((size_t)warp * MAXB + b) * (kLmax * 3) + l0 * 3 + lane] = r;
    }
    chunk_release(c);
  }
  csync();
  // sigmoid gates; transmit gate of position t into rg_hist
  for (int i = tid; i < B * L; i += kCons) {
    const int b = i / L, l = i - b * L;
    float pre[3];
#pragma unroll
    for (int g = 0; g < 3; ++g) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += red[((size_t)w * MAXB + b) * (kLmax * 3) + l * 3 + g];
      pre[g] = s + lp.b_gates[((size_t)h * L + l) * 3 + g];
    }
    const float okf = t - (1ll << l) >= 0 ? 1.f : 0.f;
    const float ig = sigmoidf_(pre[0]) * okf;
    const float fg = sigmoidf_(pre[1]) * okf + (1.f - okf);
    const float rgt = sigmoidf_(pre[2]);
    if (c.hpart == 0) rg[(((size_t)b * ml + t) * L + l) * H + h] = f2bf(rgt);
    s_f[b * kLmax + l] = fg;
    s_c[b * kLmax + l] = ig * s_rg[b * kLmax + l];
  }
  csync();
  // level recurrence (fp32 state, every level's value stored into its ring;
  // the head's two CTAs compute the same values, the first one stores them)
  for (int i = tid; i < B * (hd / 8); i += kCons) {
    const int b = i / (hd / 8), g = i - b * (hd / 8);
    const int c0 = h * hd + g * 8;
    __nv_bfloat16* ringb = ring + (size_t)b * S * d;
    const bool wr = c.hpart == 0;
    float V[8];
    const uint4 v0 = s_v0[b * 8 + g];
    unpack8(v0, V);
    if (wr) *reinterpret_cast<uint4*>(ringb + (size_t)(t & 1) * d + c0) = v0;  // ring 0 at t
#pragma unroll 4
    for (int l = 0; l < kLmax; ++l) {
      if (l < L) {
        float vs[8];
        unpack8(*reinterpret_cast<const uint4*>(s_ring + ((size_t)b * kLmax + l) * 64 + g * 8), vs);
        const float f = s_f[b * kLmax + l], cc = s_c[b * kLmax + l];
#pragma unroll
        for (int j = 0; j < 8; ++j) V[j] = f * V[j] + cc * vs[j];
        if (wr && l + 1 < L) {
          const long long slot = ((2ll << (l + 1)) - 2) + (t & ((2ll << (l + 1)) - 1));
          *reinterpret_cast<uint4*>(ringb + (size_t)slot * d + c0) = pack8(V);
        }
      }
    }
    const uint4 yv = pack8(V);
    float yr[8];
    unpack8(yv, yr);  // y is bf16, as the reference's
#pragma unroll
    for (int j = 0; j < 8; ++j) s_y[b * 64 + g * 8 + j] = yr[j];
  }
  csync();
  // out-projection share: x[b, n] += sum_c W_out[n, h*hd + c] y_h[b, c] for this
  // CTA's half of the rows n, added into both residual buffers.  Thread r owns
  // row r of a chunk (256 rows x 64 channels), reading its 16-byte pieces in a
  // rotated order (no bank conflicts); four rows leave in one vector reduction.
  const Seg so = get_seg(c, li, PH_B, 1);
  const int upc = units_per_chunk(c, so);
  const int nbase = c.hpart * (d / kHeadParts);
  for (int cu = 0; cu < so.units; cu += upc) {
    const int nrows = min(upc, so.units - cu) * 32;
    const uint8_t* chunk = chunk_acquire(c);
    const int r = tid;
    float sum[MAXB];
#pragma unroll
    for (int b = 0; b < MAXB; ++b) sum[b] = 0.f;
    if (r < nrows) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
      uint4 wv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        wv[i] = *reinterpret_cast<const uint4*>(chunk + ((size_t)r * 64 + ((half * 4 + i + r) & 7) * 8) * 2);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int pc = (half * 4 + i + r) & 7;
        float wf[8];
        unpack8(wv[i], wf);
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          if (b < B) {
            const float4 y0 = *reinterpret_cast<const float4*>(s_y + b * 64 + pc * 8);
            const float4 y1 = *reinterpret_cast<const float4*>(s_y + b * 64 + pc * 8 + 4);
            sum[b] = fmaf(wf[0], y0.x, fmaf(wf[1], y0.y, fmaf(wf[2], y0.z, fmaf(wf[3], y0.w,
                     fmaf(wf[4], y1.x, fmaf(wf[5], y1.y, fmaf(wf[6], y1.z, fmaf(wf[7], y1.w, sum[b]))))))));
          }
        }
      }
      }
    }
    const int n = nbase + cu * 32 + r;
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < B) {
        const float s1 = __shfl_down_sync(0xffffffffu, sum[b], 1);
        const float s2 = __shfl_down_sync(0xffffffffu, sum[b], 2);
        const float s3 = __shfl_down_sync(0xffffffffu, sum[b], 3);
        if ((lane & 3) == 0 && r < nrows) {
          red_add_v4(c.p.x + (size_t)b * d + n, sum[b], s1, s2, s3);
          red_add_v4(c.p.x_in + (size_t)b * d + n, sum[b], s1, s2, s3);
        }
      }
    }
    chunk_release(c);
  }
  stamp(c, li, PH_B, 3);
  grid_arrive(c, li, PH_B);
}

// GEMV CTAs: split-window attention with last-arriver combine
template <int MAXB>
__device__ void phase_b_attn(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  constexpr int HD = 64;
  const int B = c.B, H = c.H, d = c.d, ns = c.nsplit;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long t = c.t;
  const int ml = c.p.max_len;
  const long long lo = c.p.window > 0 ? (t + 1 - c.p.window > 0 ? t + 1 - c.p.window : 0) : 0;
  const long long n = t + 1 - lo;
  const long long chunk = (n + ns - 1) / ns;
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(lp.k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(lp.v_cache);
  const int items = B * H * ns;
  float* sq = c.misc;            // [64]
  float* sred = sq + 64;         // [8]
  float* sacc = sred + 8;        // [kWarps][64]
  int* flag = reinterpret_cast<int*>(sacc + kWarps * 64);
  float* sc = reinterpret_cast<float*>(flag + 4);  // scores [chunk]
  // the first item's earlier positions go to shared memory before the wait
  const int first = c.cta;
  if (first < items) {
    const int b = first / (H * ns), h = (first / ns) % H, split = first % ns;
    const long long s0 = lo + split * chunk;
    long long s1 = s0 + chunk;
    if (s1 > t) s1 = t;  // position t is written in phase A of this step
    const int cnt = s1 > s0 ? (int)min((long long)kKvPos, s1 - s0) : 0;
    for (int i = tid; i < cnt * 16; i += kCons) {
      const int pos = i >> 4, part = i & 15, kvsel = part >> 3, g = part & 7;
      const __nv_bfloat16* src = (kvsel ? vc : kc) + ((size_t)b * ml + s0 + pos) * d + h * HD + g * 8;
      cp_async16(c.kv + ((size_t)kvsel * kKvPos + pos) * HD + g * 8, src);
    }
  }
  stamp(c, li, PH_B, 0);
  grid_wait(c, li, PH_A, c.NG);
  stamp(c, li, PH_B, 1);
  cp_async_wait_all();
  csync();
  stamp(c, li, PH_B, 2);
  const float scale = rsqrtf((float)HD);
  for (int item = first; item < items; item += c.NG) {
    const int b = item / (H * ns), h = (item / ns) % H, split = item % ns;
    const long long s0 = lo + split * chunk;
    long long s1 = s0 + chunk;
    if (s1 > t + 1) s1 = t + 1;
    const int cnt = s1 > s0 ? (int)(s1 - s0) : 0;
    const int staged = item == first ? (int)min((long long)kKvPos, max(0ll, min(s1, t) - s0)) : 0;
    if (tid < HD) sq[tid] = bf2f(__ldcg(static_cast<const __nv_bfloat16*>(c.p.q) + (size_t)b * d + h * HD + tid));
    csync();
    float mloc = -INFINITY;
    for (int i = tid; i < cnt; i += kCons) {
      const __nv_bfloat16* kr = i < staged ? c.kv + (size_t)i * HD
                                           : kc + ((size_t)b * ml + s0 + i) * d + h * HD;
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < HD / 8; ++j) {
        float f[8];
        unpack8(i < staged ? reinterpret_cast<const uint4*>(kr)[j] : __ldcg(reinterpret_cast<const uint4*>(kr) + j), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(f[e], sq[j * 8 + e], s);
      }
      s *= scale;
      sc[i] = s;
      mloc = fmaxf(mloc, s);
    }
    mloc = warp_max(mloc);
    if (lane == 0) sred[warp] = mloc;
    csync();
    float M = sred[0];
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, sred[w]);
    csync();
    float lsum = 0.f;
    for (int i = tid; i < cnt; i += kCons) {
      const float e = expf(sc[i] - M);
      sc[i] = e;
      lsum += e;
    }
    lsum = warp_sum(lsum);
    if (lane == 0) sred[warp] = lsum;
    csync();
    float Ls = 0.f;
    for (int w = 0; w < kWarps; ++w) Ls += sred[w];
    const int c2 = lane * 2;
    float a0 = 0.f, a1 = 0.f;
    for (int i = warp; i < cnt; i += kWarps) {
      const __nv_bfloat162 vv =
          i < staged ? *reinterpret_cast<const __nv_bfloat162*>(c.kv + ((size_t)kKvPos + i) * HD + c2)
                     : __ldcg(reinterpret_cast<const __nv_bfloat162*>(vc + ((size_t)b * ml + s0 + i) * d + h * HD + c2));
      const float2 f = __bfloat1622float2(vv);
      a0 = fmaf(sc[i], f.x, a0);
      a1 = fmaf(sc[i], f.y, a1);
    }
    sacc[warp * HD + c2] = a0;
    sacc[warp * HD + c2 + 1] = a1;
    csync();
    float* mine = c.p.part + (((size_t)b * H + h) * ns + split) * (HD + 2);
    if (tid < HD) {
      float o = 0.f;
      for (int w = 0; w < kWarps; ++w) o += sacc[w * HD + tid];
      mine[2 + tid] = o;
    }
    if (tid == 0) {
      mine[0] = cnt > 0 ? M : -INFINITY;
      mine[1] = cnt > 0 ? Ls : 0.f;
    }
    __threadfence();
    csync();
    if (tid == 0) *flag = (atomicAdd(&c.p.counters[H + b * H + h], 1) == ns - 1);
    csync();
    if (*flag) {
      __threadfence();
      const float* all = c.p.part + ((size_t)b * H + h) * ns * (HD + 2);
      float Mx = -INFINITY;
      for (int s = 0; s < ns; ++s) Mx = fmaxf(Mx, __ldcg(all + s * (HD + 2)));
      if (tid < HD) {
        float num = 0.f, den = 0.f;
        for (int s = 0; s < ns; ++s) {
          const float ms = __ldcg(all + s * (HD + 2));
          if (ms == -INFINITY) continue;
          const float w = expf(ms - Mx);
          den += w * __ldcg(all + s * (HD + 2) + 1);
          num += w * __ldcg(all + s * (HD + 2) + 2 + tid);
        }
        static_cast<__nv_bfloat16*>(c.p.y)[(size_t)b * d + h * HD + tid] = f2bf(den > 0.f ? num / den : 0.f);
      }
      if (tid == 0) c.p.counters[H + b * H + h] = 0;
      // this (row, head) is complete: one arrival of phase B
      grid_arrive(c, li, PH_B);
    }
    csync();
  }
}

// GEMV CTAs: attention output projection, rows owned (no atomics)
template <int MAXB>
__device__ void phase_o(Ctx& c, int li) {
  const int d = c.d;
  stamp(c, li, PH_O, 0);
  grid_wait(c, li, PH_B, c.B * c.H);
  stamp(c, li, PH_O, 1);
  stage_copy(c, static_cast<const __nv_bfloat16*>(c.p.y), d);
  stamp(c, li, PH_O, 2);
  int u0, u1;
  split_range(d / 2, c.NG, c.cta, u0, u1);
  const Seg s = get_seg(c, li, PH_O, 0);
  float* x = c.p.x;
  float* xin = c.p.x_in;
  gemv_segment<MAXB>(c, s, d, u0, [&](int u, int b, int row, float v, float) {
    const size_t i = (size_t)b * d + 2 * u + row;
    const float nx = __ldcg(x + i) + v;
    x[i] = nx;
    xin[i] = nx;
  });
  stamp(c, li, PH_O, 3);
  grid_arrive(c, li, PH_O);
}

// GEMV CTAs: the FFN slice, down projection added into x
template <int MAXB>
__device__ void phase_c(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  const int d = c.d, B = c.B, tid = threadIdx.x;
  stamp(c, li, PH_C, 0);
  if (lp.kind == 0) grid_wait(c, li, PH_B, c.H * kHeadParts);
  else grid_wait(c, li, PH_O, c.NG);
  stamp(c, li, PH_C, 1);
  stage_norm<MAXB>(c, c.p.x_in, static_cast<const __nv_bfloat16*>(lp.norm2));
  stamp(c, li, PH_C, 2);
  int j0, j1;
  split_range(c.ff, c.NG, c.cta, j0, j1);
  float* us = c.misc;  // [MAXB][kMaxUpc]
  const Seg sgu = get_seg(c, li, PH_C, 0);
  gemv_segment<MAXB>(c, sgu, d, 0, [&](int u, int b, int row, float g, float up) {
    if (row != 0) return;
    us[b * kMaxUpc + u] = bf2f(f2bf(g / (1.0f + expf(-g)) * up));
  });
  csync();
  const Seg sd = get_seg(c, li, PH_C, 1);
  const int upc = units_per_chunk(c, sd);
  const int n0 = tid * 4;
  const bool nin = n0 < d;
  float acc[MAXB][4];
#pragma unroll
  for (int b = 0; b < MAXB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = acc[b][3] = 0.f;
  for (int cu = 0; cu < sd.units; cu += upc) {
    const int nj = min(upc, sd.units - cu);
    const uint8_t* chunk = chunk_acquire(c);
    if (nin) {
#pragma unroll 4
      for (int j = 0; j < nj; ++j) {
        const uint2 wv = *reinterpret_cast<const uint2*>(chunk + ((size_t)j * d + n0) * 2);
        const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.x));
        const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.y));
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          if (b < B) {
            const float uj = us[b * kMaxUpc + cu + j];
            acc[b][0] = fmaf(uj, w01.x, acc[b][0]);
            acc[b][1] = fmaf(uj, w01.y, acc[b][1]);
            acc[b][2] = fmaf(uj, w23.x, acc[b][2]);
            acc[b][3] = fmaf(uj, w23.y, acc[b][3]);
          }
        }
      }
    }
    chunk_release(c);
  }
  if (nin && sd.units > 0) {
#pragma unroll
    for (int b = 0; b < MAXB; ++b)
      if (b < B) red_add_v4(c.p.x + (size_t)b * d + n0, acc[b][0], acc[b][1], acc[b][2], acc[b][3]);
  }
  stamp(c, li, PH_C, 3);
  grid_arrive(c, li, PH_C);
}

template <int MAXB>
__device__ void phase_n(Ctx& c) {
  const int d = c.d, nl = c.p.n_layers;
  stamp(c, nl, 0, 0);
  grid_wait(c, nl - 1, PH_C, c.NG);
  stamp(c, nl, 0, 1);
  stage_norm<MAXB>(c, c.p.x, static_cast<const __nv_bfloat16*>(c.p.norm_out));
  stamp(c, nl, 0, 2);
  int u0, u1;
  split_range((c.p.vocab + 1) / 2, c.G, c.cta, u0, u1);
  const Seg s = get_seg(c, c.p.n_layers, PH_N, 0);
  __nv_bfloat16* lg = static_cast<__nv_bfloat16*>(c.p.logits);
  const int V = c.p.vocab;
  gemv_segment<MAXB>(c, s, d, u0, [&](int u, int b, int row, float v, float) {
    lg[(size_t)b * V + 2 * u + row] = f2bf(v);
  });
  stamp(c, nl, 0, 3);
}

// ------------------------------------------------------------------ kernel
template <int MAXB>
__global__ void __launch_bounds__(kThreads, 1)
    step_kernel(const __grid_constant__ dh_step_params p, uint32_t wait_limit) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Ctx c{p};
  c.G = gridDim.x;
  c.cta = blockIdx.x;
  c.B = p.batch;
  c.d = p.d;
  c.gh = p.d;
  c.L = p.L;
  c.H = p.H;
  c.hd = p.hd;
  c.ff = p.ff;
  c.NG = c.G - c.H * kHeadParts;
  c.head = c.cta >= c.NG ? (c.cta - c.NG) / kHeadParts : -1;
  c.hpart = c.cta >= c.NG ? (c.cta - c.NG) % kHeadParts : 0;
  c.wait_limit = wait_limit;
  {
    int ns = c.NG / (c.B * c.H);
    ns = ns < 1 ? 1 : ns;
    c.nsplit = ns < p.nsplit ? ns : p.nsplit;
  }
  c.lg = 1;
  while (c.lg < c.L && c.lg < kLgMax && gate_chunk_bytes(c, 0, c.lg + 1) <= (uint32_t)kSlotBytes)
    ++c.lg;
  c.nslots = slots_for<MAXB>();
  c.slots = smem_raw;
  uint8_t* q = smem_raw + (size_t)c.nslots * kSlotBytes;
  c.xs = reinterpret_cast<__nv_bfloat16*>(q);
  q += (size_t)MAXB * 1024 * 2;
  c.kv = reinterpret_cast<__nv_bfloat16*>(q);
  q += (size_t)2 * kKvPos * 64 * 2;
  c.red = reinterpret_cast<float*>(q);
  q += (size_t)kWarps * MAXB * kLmax * 3 * 4;
  c.misc = reinterpret_cast<float*>(q);
  q += (size_t)(MAXB * (4 * kLmax + 64 + kMaxUpc) + MAXB * kLmax * 32 + 2048) * 4;
  static_assert(3 * kLmax + 64 + 32 + kLmax * 32 <= 4 * kLmax + 64 + kMaxUpc + kLmax * 32,
                "head phase arrays fit the per-row scratch");
  c.full = reinterpret_cast<uint64_t*>(q);
  c.empty = c.full + c.nslots;
  c.abort = reinterpret_cast<volatile int*>(c.empty + c.nslots);
  c.consumed = 0;
  c.t = __ldcg(p.t_buf);
  c.gen = __ldcg(p.barrier);
  if (c.t < 0 || c.t >= p.max_len) {  // no position left: nothing is written
    if (c.cta == 0 && threadIdx.x == 0) atomicExch(p.status, DH_ERR_ARG);
    return;
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < c.nslots; ++s) {
      mbar_init(&c.full[s], 1);
      mbar_init(&c.empty[s], kWarps);
    }
    *c.abort = 0;
    fence_barrier_init();
  }
  c.prod = reinterpret_cast<Prod*>(const_cast<int*>(reinterpret_cast<volatile int*>(c.abort)) + 4);
  {  // the layer table, read once into shared memory
    dh_layer_params* lay = reinterpret_cast<dh_layer_params*>(
        reinterpret_cast<uint8_t*>(c.prod) + ((sizeof(Prod) + 15) / 16) * 16);
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.layers);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(lay);
    const int words = p.n_layers * (int)(sizeof(dh_layer_params) / 8);
    for (int i = threadIdx.x; i < words; i += kThreads) dst[i] = src[i];
    c.lay = lay;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Prod* pr = c.prod;
    pr->pp = &p;
    pr->lay = c.lay;
    pr->emb = p.emb;
    pr->vocab = p.vocab;
    pr->max_len = p.max_len;
    pr->n_layers = p.n_layers;
    pr->G = c.G; pr->cta = c.cta; pr->NG = c.NG; pr->head = c.head; pr->hpart = c.hpart;
    pr->B = c.B; pr->d = c.d; pr->gh = c.gh; pr->L = c.L; pr->H = c.H; pr->hd = c.hd;
    pr->ff = c.ff; pr->lg = c.lg; pr->nslots = c.nslots; pr->t = c.t;
    pr->wait_limit = c.wait_limit;
    pr->slots = c.slots; pr->full = c.full; pr->empty = c.empty; pr->abort = c.abort;
    pr->issued = 0; pr->pslot = 0; pr->peph = 0;
    cursor_seek(pr, 0, 0, 0);
  }
  __syncthreads();
  stamp(c, p.n_layers, 1, 0);
  if (threadIdx.x >= kCons) {  // the producer warpgroup: one lane works, the rest leave
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kProdRegs));
    if (threadIdx.x == kCons) producer(c.prod, p.status);
    return;
  }
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kConsRegs));
  const int nl = p.n_layers;
  for (int li = 0; li < nl; ++li) {
    const bool tree = c.lay[li].kind == 0;
    if (c.head < 0) {
      phase_a<MAXB>(c, li);
      if (tree) {
        phase_c<MAXB>(c, li);
      } else {
        phase_b_attn<MAXB>(c, li);
        phase_o<MAXB>(c, li);
        phase_c<MAXB>(c, li);
      }
    } else if (tree) {
      phase_b_tree<MAXB>(c, li);
    }
  }
  phase_n<MAXB>(c);
  cp_async_wait_all();
  stamp(c, p.n_layers, 1, 1);
  if (c.cta == 0 && threadIdx.x == 0) {
    p.t_buf[0] = c.t + 1;
    atomicAdd(p.barrier, 1ull);
  }
}

template <int MAXB>
size_t step_smem() {
  return (size_t)slots_for<MAXB>() * kSlotBytes + (size_t)MAXB * 1024 * 2 + (size_t)2 * kKvPos * 64 * 2 +
         (size_t)kWarps * MAXB * kLmax * 3 * 4 +
         (size_t)(MAXB * (4 * kLmax + 64 + kMaxUpc) + MAXB * kLmax * 32 + 2048) * 4 +
         (size_t)2 * slots_for<MAXB>() * 8 + 64 + ((sizeof(Prod) + 15) / 16) * 16 +
         (size_t)kMaxLayers * sizeof(dh_layer_params);
}

template <int MAXB>
int launch_step(const dh_step_params& p, cudaStream_t st) {
  const size_t smem = step_smem<MAXB>();
  DH_REQUIRE(smem <= 227 * 1024, DH_ERR_SHAPE, "dh_decode_step: %zu bytes of shared memory", smem);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(step_kernel<MAXB>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured_dev = dev;
  }
  int per_sm = 0;
  const cudaError_t occ =
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel<MAXB>, kThreads, smem);
  if (per_sm < 1) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, step_kernel<MAXB>);
    return set_error(DH_ERR_SHAPE,
                     "dh_decode_step: kernel does not fit on an SM (%s; %d regs, %zu B smem "
                     "requested, max dynamic %d, max threads %d)",
                     cudaGetErrorString(occ), fa.numRegs, smem, fa.maxDynamicSharedSizeBytes,
                     fa.maxThreadsPerBlock);
  }
  const int G = sm_count();
  DH_REQUIRE(G - p.H * kHeadParts >= 16, DH_ERR_SHAPE,
             "dh_decode_step: %d SMs leave too few GEMV CTAs", G);
  {  // the attention scores of one item live in the per-phase scratch
    const int span = (p.window > 0 && p.window < p.max_len) ? p.window : p.max_len;
    int ns = (G - p.H * kHeadParts) / (p.batch * p.H);
    ns = ns < 1 ? 1 : (ns < p.nsplit ? ns : p.nsplit);
    const int chunk = (span + ns - 1) / ns;
    const int misc = MAXB * (4 * kLmax + 64 + kMaxUpc) + MAXB * kLmax * 32 + 2048;
    DH_REQUIRE(chunk + 64 + 8 + kWarps * 64 + 4 <= misc, DH_ERR_SHAPE,
               "dh_decode_step: %d window positions per attention item exceed the scratch", chunk);
  }
  DH_REQUIRE((p.ff + (G - p.H * kHeadParts) - 1) / (G - p.H * kHeadParts) <= kMaxUpc,
             DH_ERR_SHAPE, "dh_decode_step: FFN width %d too large for %d CTAs", p.ff,
             G - p.H * kHeadParts);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, step_kernel<MAXB>, p, wait_limit()) != cudaSuccess)
    return check_launch("step_kernel");
  return DH_OK;
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_decode_step(const dh_step_params* params, void* stream) {
  DH_REQUIRE(params, DH_ERR_ARG, "dh_decode_step: null params");
  const dh_step_params& p = *params;
  DH_REQUIRE(p.layers && p.tokens && p.t_buf && p.emb && p.norm_out && p.logits && p.x && p.x_in &&
                 p.a && p.v0 && p.y && p.q && p.part && p.counters && p.barrier && p.status,
             DH_ERR_ARG, "dh_decode_step: null pointer in params");
  DH_REQUIRE(p.batch >= 1 && p.batch <= 8, DH_ERR_SHAPE, "dh_decode_step: batch %d not in [1,8]",
             p.batch);
  DH_REQUIRE(p.hd == 64 && p.d == p.H * p.hd && p.d % 64 == 0 && p.d <= 1024 && p.ff % 8 == 0 &&
                 p.L >= 1 && p.L <= kLmax && p.nsplit >= 1 && p.n_layers >= 1 &&
                 p.n_layers <= kMaxLayers,
             DH_ERR_SHAPE, "dh_decode_step: unsupported shape (d=%d H=%d hd=%d ff=%d L=%d layers=%d)",
             p.d, p.H, p.hd, p.ff, p.L, p.n_layers);
  DH_REQUIRE(4 * p.d <= kSlotBytes && 3 * p.d * 2 + p.batch * p.d * 2 <= kSlotBytes, DH_ERR_SHAPE,
             "dh_decode_step: a weight unit exceeds a stream slot (d=%d batch=%d)", p.d, p.batch);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.batch == 1) return launch_step<1>(p, st);
  if (p.batch == 2) return launch_step<2>(p, st);
  if (p.batch <= 4) return launch_step<4>(p, st);
  return launch_step<8>(p, st);
}
