// Whole decode step as ONE persistent cooperative kernel (one CTA per SM).
//
// Roles.  The last 2H CTAs are "head" CTAs (two per attention head of the
// mixer); the others are "GEMV" CTAs.  A tree block is three dependent
// phases:
//   A  (GEMV CTAs)  h = RMSNorm(x); [v0 | A | B_hist[t]] = W3 h
//   B  (head CTAs)  head h: the gate readouts of all levels
//                   (W_l . relu^2(A + B_hist[t - 2^l])), the level recurrence
//                   over the ring buffers, and half of the head's share of the
//                   output projection, added into the residual
//   C  (GEMV CTAs)  h2 = RMSNorm(x); u = silu(Wg h2) * (Wu h2) for this CTA's
//                   slice of the FFN width; x += Wd[:, slice] u
// An attention block is A (q, k, v with RoPE, cache write), B (window
// attention split over the GEMV CTAs, last-arriver combine), O (output
// projection, rows owned) and C.  The step ends with the logits on all CTAs.
// This follows the reference's fused step (decoding.py:457-488 with
// fused_step.py:26-88) and attention step (decoding.py:411-435).
//
// Arithmetic.  Every weight contraction runs on the tensor cores as
// mma.sync.m16n8k16 (bf16 operands from shared memory through ldmatrix, fp32
// accumulators): a CUDA-core dot product needs ~17 instructions per 16 bytes
// of bf16 weights (load, eight conversions, eight FMAs), which caps a whole
// step at ~550 us on 148 SMs, while one mma consumes 512 bytes of weights.
// The N = 8 columns of an mma hold the lockstep rows.  tcgen05.mma is not used
// here: a CTA owns only a few 16-row tiles of each matrix and a tcgen05
// instruction costs ~120-130 cycles whatever its N, so a 1024-wide row block
// would take >= 64 instructions (~4 us) per phase.  K is split over the 8
// consumer warps; their partial tiles meet in shared memory.  Weights are
// stored in HBM with the 16-byte chunks of every row XOR-permuted by
// (row & 7) (packed once by the host), so a linear bulk copy lands them in a
// layout whose ldmatrix reads are free of bank conflicts.
//
// Streaming.  Weights never depend on activations, so each CTA's producer
// lane streams its slices of every phase of the step, in consumption order,
// by bulk async copies (cp.async.bulk) into a ring of shared-memory slots
// that runs ahead of the phase waits; history rows the head CTAs need
// (B_hist at t - 2^l) travel in the same stream, and ring slots, transmit
// gates at the source positions and the attention window's keys and values
// (all written by earlier steps) are loaded before each wait.  After a wait
// a phase reads only the small activation vector and computes from shared
// memory.
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
constexpr int kSlots = 5;
constexpr int kMaxB = 2;                     // lockstep rows of this kernel
constexpr int kKvPos = 128;                  // window positions staged per attention item
constexpr int kHeadParts = 2;                // head CTAs per head (each takes half the out-projection rows)
constexpr int kLmax = 16;
constexpr int kMaxUpc = 32;                  // FFN elements per GEMV CTA
constexpr int kMaxD = 1024;
constexpr int kMisc = 4096;                  // floats of per-phase scratch
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
__device__ __forceinline__ void red_add_f32(float* p, float a) {
  asm volatile("red.global.add.f32 [%0], %1;" ::"l"(p), "f"(a) : "memory");
}
__device__ __forceinline__ void red_add_v2(float* p, float a, float b) {
  asm volatile("red.global.add.v2.f32 [%0], {%1, %2};" ::"l"(p), "f"(a), "f"(b) : "memory");
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

// tensor-core fragments (m16n8k16, bf16 in, fp32 accumulate)
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x2_t(uint32_t (&r)[2], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
               : "=r"(r[0]), "=r"(r[1])
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], const uint32_t (&b)[2]) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
}
// byte offset of 16-byte chunk `ch` of row `r` in a swizzled tile of rows of `rb` bytes
__device__ __forceinline__ uint32_t swz(int r, int ch, int rb) {
  return (uint32_t)(r * rb + ((ch ^ (r & 7)) << 4));
}

// ------------------------------------------------------------------ the plan
// A segment is a run of equal units of one matrix (or of history rows) that
// this CTA streams for one phase; a chunk is up to one slot of whole units.
enum { SEG_ROWS = 0, SEG_BHIST = 1 };
struct Seg {
  const uint8_t* base;
  uint32_t unit_bytes;
  int units;
  int kind;
  size_t limit;   // bytes readable from base (the last unit may be short)
  int per_chunk;  // units per chunk
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
  int nslots;            // ring slots
  // shared memory
  uint8_t* slots;
  uint64_t* full;
  uint64_t* empty;
  volatile int* abort;
  __nv_bfloat16* xs;     // staged activation rows [kMaxB][kMaxD], chunk-swizzled
  __nv_bfloat16* zrow;   // a row of zeros (kMaxD)
  float* red;            // partial tiles / reductions
  float* misc;           // small per-phase arrays
  __nv_bfloat16* kv;     // [2][kKvPos][hd]
  int acq, rel;          // chunks acquired / released (same in every consumer thread)
  struct Prod* prod;     // the weight stream (shared memory; the producer lane)
  const dh_layer_params* lay;  // the layer table, copied into shared memory
};

// The weight stream's state, in shared memory, used by the producer lane: a
// copy of the CTA's geometry and the cursor of the next chunk.
struct Prod {
  const dh_layer_params* lay;
  const void* lm_head;
  int vocab, max_len, n_layers;
  int G, cta, NG, head, hpart, B, d, gh, L, H, hd, ff, nslots;
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

// the few step parameters the plan needs, for the consumers' context and for
// the issuer's shared-memory copy
__device__ __forceinline__ int vocab_of(const Ctx& c) { return c.p.vocab; }
__device__ __forceinline__ int vocab_of(const Prod& c) { return c.vocab; }
__device__ __forceinline__ const void* lm_head_of(const Ctx& c) { return c.p.lm_head; }
__device__ __forceinline__ const void* lm_head_of(const Prod& c) { return c.lm_head; }

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

// bytes between two history rows in a B_hist chunk: one 16-byte chunk more
// than a row, so the rows of an ldmatrix read fall in different banks
template <class C>
__device__ __forceinline__ int bh_stride(const C& c) { return c.gh * 2 + 16; }

// number of segments of (layer li, phase ph) for this CTA, and segment si
template <class C>
__device__ int seg_count(const C& c, int li, int ph) {
  if (ph == PH_N) return 1;
  const bool tree = layer(c, li).kind == 0;
  if (c.head >= 0) return (tree && ph == PH_B) ? 3 : 0;
  if (ph == PH_A || ph == PH_O) return (ph == PH_O && tree) ? 0 : 1;
  if (ph == PH_C) return 2;
  return 0;
}

template <class C>
__device__ Seg get_seg(const C& c, int li, int ph, int si) {
  Seg s{nullptr, 1, 0, SEG_ROWS, 0, 1};  // one tile per chunk unless stated
  const int d = c.d;
  if (ph == PH_N) {  // 16-row tiles of the (swizzled) lm_head, split over every CTA
    const int V = vocab_of(c);
    int u0, u1;
    split_range((V + 15) / 16, c.G, c.cta, u0, u1);
    s.base = static_cast<const uint8_t*>(lm_head_of(c)) + (size_t)u0 * 32 * d;
    s.unit_bytes = 32 * d;
    s.units = u1 - u0;
    s.limit = (size_t)V * d * 2 - (size_t)u0 * 32 * d;
    return s;
  }
  const dh_layer_params& lp = layer(c, li);
  if (c.head >= 0) {  // tree block B: history rows, gate readout tiles, out-projection rows
    if (si == 0) {
      s.base = static_cast<const uint8_t*>(lp.b_hist);
      s.unit_bytes = (uint32_t)(c.L * bh_stride(c));  // one lockstep row's L history rows
      s.units = c.B;
      s.kind = SEG_BHIST;
    } else if (si == 1) {  // three 16-row tiles: admit, forget, transmit rows of every level
      s.base = static_cast<const uint8_t*>(lp.w_gates) + (size_t)c.head * 3 * 16 * c.gh * 2;
      s.unit_bytes = 16 * c.gh * 2;
      s.units = 3;
    } else {  // this CTA's half of the output rows, head h's columns
      s.base = static_cast<const uint8_t*>(lp.w_out) +
               ((size_t)c.head * d + (size_t)c.hpart * (d / kHeadParts)) * c.hd * 2;
      s.unit_bytes = 16 * c.hd * 2;  // one 16-row tile
      s.units = d / kHeadParts / 16;
      s.per_chunk = kSlotBytes / (16 * c.hd * 2);
    }
    s.limit = (size_t)s.units * s.unit_bytes;
    return s;
  }
  const int gi = c.cta;
  int u0, u1;
  if (ph == PH_A || ph == PH_O) {  // 16-row tiles of W3 / Wqkv / W_out
    const int units = ph == PH_A ? 3 * d / 16 : d / 16;
    split_range(units, c.NG, gi, u0, u1);
    s.base = static_cast<const uint8_t*>(ph == PH_A ? lp.w_in3 : lp.w_out) + (size_t)u0 * 32 * d;
    s.unit_bytes = 32 * d;
    s.units = u1 - u0;
    s.limit = (size_t)s.units * s.unit_bytes;
  } else {  // PH_C: 16-row tiles of (gate, up) row pairs (8 FFN columns each), then Wd^T rows
    split_range(c.ff / 8, c.NG, gi, u0, u1);
    if (si == 0) {
      s.base = static_cast<const uint8_t*>(lp.w_gu) + (size_t)u0 * 32 * d;
      s.unit_bytes = 32 * d;
      s.units = u1 - u0;
      s.limit = (size_t)s.units * s.unit_bytes;
    } else {  // 16-row tiles of Wd^T over the same 8 (u1 - u0) FFN columns
      const int jn = 8 * (u1 - u0);
      s.base = static_cast<const uint8_t*>(lp.w_down) + (size_t)u0 * 8 * 2 * d;
      s.unit_bytes = 32 * d;
      s.units = (jn + 15) / 16;
      s.limit = (size_t)jn * 2 * d;
    }
  }
  return s;
}

template <class C>
__device__ __forceinline__ int units_per_chunk(const C&, const Seg& s) { return s.per_chunk; }

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
  if (s.kind == SEG_BHIST) {  // lockstep row u: its history rows of every level
    const int gh = pr->gh, L = pr->L, stride = bh_stride(*pr);
    const long long t = pr->t;
    uint32_t total = 0;
    for (int l = 0; l < L; ++l)
      if (t - (1ll << l) >= 0) total += (uint32_t)gh * 2;
    mbar_arrive_expect_tx(bar, total);
    const __nv_bfloat16* bh = reinterpret_cast<const __nv_bfloat16*>(s.base);
    for (int l = 0; l < L; ++l) {
      const long long src = t - (1ll << l);
      if (src < 0) continue;
      bulk_g2s(dst + (size_t)l * stride, bh + ((size_t)u * pr->max_len + src) * gh, (uint32_t)gh * 2,
               bar);
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

// The producer (one lane of the producer warpgroup): walks the plan, waiting
// (bounded) for each slot to be released by every consumer warp before
// refilling it; stops at the first failed wait or when a consumer aborted,
// and finally waits (with a fixed bound) for the copies it issued.
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
// Chunks are acquired and released in stream order; a phase may hold several.
__device__ __forceinline__ const uint8_t* chunk_acquire(Ctx& c) {
  const int k = c.acq++;
  const int slot = k % c.nslots;
  if (!*c.abort) {
    if (!mbar_wait(&c.full[slot], (uint32_t)((k / c.nslots) & 1), c.p.status, c.wait_limit))
      *c.abort = 1;
  }
  return c.slots + (size_t)slot * kSlotBytes;
}

__device__ __forceinline__ void chunk_release(Ctx& c) {
  __syncwarp();
  if ((threadIdx.x & 31) == 0) mbar_arrive(&c.empty[c.rel % c.nslots]);
  c.rel += 1;
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

// xs row b, element k (a row is kMaxD wide, its 16-byte chunks XOR-permuted by b)
__device__ __forceinline__ __nv_bfloat16* xs_at(const Ctx& c, int b, int k) {
  return c.xs + (size_t)b * kMaxD + (((k >> 3) ^ (b & 7)) << 3) + (k & 7);
}

// xs[b][k] = bf16(x[b][k] * rsqrt(mean(x[b]^2) + eps) * w[k]) for every lockstep row;
// x comes from `xf` (fp32, read through L2) or, for the first block, from the
// embedding rows of the step's tokens.  The same loads also write this CTA's
// slice [e0, e1) (float4 units) of x into dst0 / dst1 when they are set.
// The norm weights this thread multiplies by, w[k..k+3] of each of its float4
// units (constant: loaded before the phase's wait).
constexpr int kNV = (kMaxB * kMaxD + kCons * 4 - 1) / (kCons * 4);
struct NormW {
  uint2 w[kNV];
};
__device__ __forceinline__ NormW load_normw(const Ctx& c, const __nv_bfloat16* w) {
  NormW nw;
  const int d4 = c.d / 4, n4 = c.B * d4;
#pragma unroll
  for (int j = 0; j < kNV; ++j) {
    const int i = threadIdx.x + j * kCons;
    nw.w[j] = i < n4 ? *reinterpret_cast<const uint2*>(w + (i - (i / d4) * d4) * 4) : make_uint2(0, 0);
  }
  return nw;
}

__device__ void stage_norm(Ctx& c, const float* xf, const NormW& nw, float* dst0 = nullptr,
                           float* dst1 = nullptr, int e0 = 0, int e1 = 0) {
  const int B = c.B, d = c.d, d4 = d / 4, n4 = B * d4;
  constexpr int NV = kNV;
  float* ssum = c.misc + kMisc - kMaxB;  // [kMaxB]
  if (threadIdx.x < kMaxB) ssum[threadIdx.x] = 0.f;
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
        if (tok < 0 || tok >= c.p.vocab) tok = 0;  // reported by phase A of the first block
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
      const uint2 wv = nw.w[j];
      const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.x));
      const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.y));
      uint2 pk;
      pk.x = pack2(v[j].x * r * w01.x, v[j].y * r * w01.y);
      pk.y = pack2(v[j].z * r * w23.x, v[j].w * r * w23.y);
      *reinterpret_cast<uint2*>(xs_at(c, b, k)) = pk;
    }
  }
  csync();
}

// xs rows = src[b][0:K] (bf16 produced by another CTA)
__device__ void stage_copy(Ctx& c, const __nv_bfloat16* src, int K) {
  const int k8 = K / 8, n = c.B * k8;
  for (int i = threadIdx.x; i < n; i += kCons) {
    const int b = i / k8, k = (i - b * k8) * 8;
    *reinterpret_cast<uint4*>(xs_at(c, b, k)) =
        __ldcg(reinterpret_cast<const uint4*>(src + (size_t)b * K + k));
  }
  csync();
}

// B fragments of the staged rows for this warp's K range: k-step i covers
// columns [(warp * ksw + i) * 16, +16); columns n of the mma are the lockstep
// rows (rows >= B read zeros)
__device__ __forceinline__ void load_xfrags(const Ctx& c, int ksw, uint32_t (&bx)[8][2]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = lane & 7, half = (lane >> 3) & 1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (i < ksw) {
      const int ch = (warp * ksw + i) * 2 + half;
      const __nv_bfloat16* row = n < c.B ? c.xs + (size_t)n * kMaxD + ((ch ^ (n & 7)) << 3)
                                         : c.zrow + (ch << 3);
      ldsm_x2(bx[i], smem_u32(row));
    }
  }
}

// One segment of 16-row tiles (one tile per chunk) against the staged rows:
// each warp contracts its K range, the partial tiles meet in shared memory,
// and threads (row pair p, lockstep row b) run epi(tile, p, b, v_even, v_odd).
template <class Epi>
__device__ void gemv_tiles(Ctx& c, const Seg& s, const uint32_t (&bx)[8][2], int ksw, Epi epi) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t4 = lane & 3;
  const int rb = c.d * 2;  // bytes of a weight row
  const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, ahalf = lane >> 4;
  for (int u = 0; u < s.units; ++u) {
    const uint8_t* chunk = chunk_acquire(c);
    const uint32_t base = smem_u32(chunk);
    // four independent accumulator chains: the k-steps do not wait on one
    // another's mma latency
    float ac[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) ac[j][0] = ac[j][1] = ac[j][2] = ac[j][3] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (i < ksw) {
        uint32_t a[4];
        ldsm_x4(a, base + swz(arow, (warp * ksw + i) * 2 + ahalf, rb));
        mma16816(ac[i & 3], a, bx[i]);
      }
    }
    float acc[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[e] = (ac[0][e] + ac[1][e]) + (ac[2][e] + ac[3][e]);
    float* pb = c.red + ((size_t)(u & 1) * kWarps + warp) * 16 * 8;  // [16 rows][8 columns]
    pb[g * 8 + 2 * t4] = acc[0];
    pb[g * 8 + 2 * t4 + 1] = acc[1];
    pb[(g + 8) * 8 + 2 * t4] = acc[2];
    pb[(g + 8) * 8 + 2 * t4 + 1] = acc[3];
    chunk_release(c);
    csync();
    if (threadIdx.x < 8 * c.B) {
      const int p = threadIdx.x / c.B, b = threadIdx.x - p * c.B;
      const float* q = c.red + (size_t)(u & 1) * kWarps * 16 * 8;
      float v0 = 0.f, v1 = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        v0 += q[(w * 16 + 2 * p) * 8 + b];
        v1 += q[(w * 16 + 2 * p + 1) * 8 + b];
      }
      epi(u, p, b, v0, v1);
    }
  }
}

// ------------------------------------------------------------------ phases
__device__ void phase_a(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  const bool tree = lp.kind == 0;
  const int d = c.d, B = c.B;
  stamp(c, li, PH_A, 0);
  const NormW nw = load_normw(c, static_cast<const __nv_bfloat16*>(lp.norm1));
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
    stage_norm(c, li == 0 ? nullptr : c.p.x, nw, li == 0 ? c.p.x : nullptr,
               (li == 0 || tree) ? c.p.x_in : nullptr, e0, e1);
  }
  stamp(c, li, PH_A, 2);
  const int ksw = d / 128;
  uint32_t bx[8][2];
  load_xfrags(c, ksw, bx);
  const Seg s = get_seg(c, li, PH_A, 0);
  int u0, u1;
  split_range(3 * d / 16, c.NG, c.cta, u0, u1);
  const long long t = c.t;
  const int ml = c.p.max_len;
  if (tree) {
    __nv_bfloat16* v0 = static_cast<__nv_bfloat16*>(c.p.v0);
    __nv_bfloat16* a = static_cast<__nv_bfloat16*>(c.p.a);
    __nv_bfloat16* bh = static_cast<__nv_bfloat16*>(lp.b_hist);
    gemv_tiles(c, s, bx, ksw, [&](int u, int p, int b, float ve, float vo) {
      const int n = (u0 + u) * 16 + 2 * p, seg = n / d, col = n - seg * d;
      const uint32_t pk = pack2(ve, vo);
      __nv_bfloat16* dst = seg == 0 ? v0 + (size_t)b * d + col
                         : seg == 1 ? a + (size_t)b * d + col
                                    : bh + ((size_t)b * ml + t) * d + col;
      *reinterpret_cast<uint32_t*>(dst) = pk;
    });
  } else {
    __nv_bfloat16* q = static_cast<__nv_bfloat16*>(c.p.q);
    __nv_bfloat16* kc = static_cast<__nv_bfloat16*>(lp.k_cache);
    __nv_bfloat16* vc = static_cast<__nv_bfloat16*>(lp.v_cache);
    const int hd = c.hd;
    const float* cosT = c.p.rope_cos;
    const float* sinT = c.p.rope_sin;
    gemv_tiles(c, s, bx, ksw, [&](int u, int p, int b, float x1, float x2) {
      const int n = (u0 + u) * 16 + 2 * p, seg = n / d, col = n - seg * d;
      float o1 = x1, o2 = x2;
      if (seg < 2) {  // rotate the pair (2j, 2j+1) of q and k at position t
        const int j = (col % hd) >> 1;
        const float cs = cosT[t * (hd / 2) + j], sn = sinT[t * (hd / 2) + j];
        o1 = x1 * cs - x2 * sn;
        o2 = x1 * sn + x2 * cs;
      }
      const uint32_t pk = pack2(o1, o2);
      __nv_bfloat16* dst = seg == 0 ? q + (size_t)b * d + col
                         : seg == 1 ? kc + ((size_t)b * ml + t) * d + col
                                    : vc + ((size_t)b * ml + t) * d + col;
      *reinterpret_cast<uint32_t*>(dst) = pk;
    });
  }
  stamp(c, li, PH_A, 3);
  grid_arrive(c, li, PH_A);
}

// head CTA: gates of every level, level recurrence, out-projection share
__device__ void phase_b_tree(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  const int B = c.B, L = c.L, H = c.H, hd = c.hd, gh = c.gh, d = c.d, h = c.head;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g4 = lane >> 2, t4 = lane & 3;
  const long long t = c.t;
  const int ml = c.p.max_len;
  const int S = (1 << (L + 1)) - 2;
  __nv_bfloat16* ring = static_cast<__nv_bfloat16*>(lp.v_ring);
  __nv_bfloat16* rg = static_cast<__nv_bfloat16*>(lp.rg_hist);
  // small arrays in c.misc
  float* s_f = c.misc;                        // [kMaxB][kLmax]
  float* s_c = s_f + kMaxB * kLmax;           // [kMaxB][kLmax]
  float* s_rg = s_c + kMaxB * kLmax;          // [kMaxB][kLmax] transmit gate at the source
  uint4* s_v0 = reinterpret_cast<uint4*>(s_rg + kMaxB * kLmax);              // [kMaxB][8]
  __nv_bfloat16* s_y = reinterpret_cast<__nv_bfloat16*>(s_v0 + kMaxB * 8);   // [kMaxB][64]
  __nv_bfloat16* s_ring = s_y + kMaxB * 64;                                  // [kMaxB][kLmax][64]
  float* red = reinterpret_cast<float*>(s_ring + kMaxB * kLmax * 64);       // [kWarps][kMaxB][48]
  float* s_bias = red + kWarps * kMaxB * 48;                                 // [kLmax][3]
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
  for (int i = tid; i < L * 3; i += kCons) s_bias[i] = lp.b_gates[(size_t)h * L * 3 + i];
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
        *reinterpret_cast<uint4*>(xs_at(c, b, k)) =
            __ldcg(reinterpret_cast<const uint4*>(a + (size_t)b * gh + k));
      } else {
        const int j = i - n, b = j / 8, g = j - b * 8;
        s_v0[b * 8 + g] = __ldcg(reinterpret_cast<const uint4*>(v0 + (size_t)b * d + h * hd + g * 8));
      }
    }
  }
  csync();
  stamp(c, li, PH_B, 2);
  // gate readouts on the tensor cores: D = W x hv with W the three 16-row
  // tiles (admit / forget / transmit rows of levels 0..15) and hv the 16
  // columns relu^2(A + B_hist[t - 2^l]) (bf16), built in registers from
  // ldmatrix fragments of the history rows; the readout of level l is the
  // diagonal element (l, l).  K is split over the warps.
  const uint8_t* bhc[kMaxB];
  for (int b = 0; b < B; ++b) bhc[b] = chunk_acquire(c);
  const uint8_t* wg[3];
  for (int g = 0; g < 3; ++g) wg[g] = chunk_acquire(c);
  const int ksw = gh / 128;
  const int bstride = bh_stride(c);
  {
    const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, ahalf = lane >> 4;
    const int brow = lane & 7, bhalf = (lane >> 3) & 1;
    const __nv_bfloat162 z2 = __floats2bfloat162_rn(0.f, 0.f);
    for (int b = 0; b < B; ++b) {
      // two accumulator sets (even / odd k-steps) halve the mma chains
      float acc2[2][3][2][4];
#pragma unroll
      for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
        for (int g = 0; g < 3; ++g)
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc2[s2][g][nt][e] = 0.f;
#pragma unroll 1
      for (int i0 = 0; i0 < ksw; i0 += 2) {
#pragma unroll
        for (int s2 = 0; s2 < 2; ++s2) {
          const int i = i0 + s2;
          if (i >= ksw) break;
          float (&acc)[3][2][4] = acc2[s2];
          const int ch = (warp * ksw + i) * 2;  // first 16-byte chunk of this k-step
          // A values at this thread's fragment columns (k = 8 ch + 2 t4, +8)
          const __nv_bfloat162 a_lo = *reinterpret_cast<const __nv_bfloat162*>(xs_at(c, b, ch * 8 + 2 * t4));
          const __nv_bfloat162 a_hi = *reinterpret_cast<const __nv_bfloat162*>(xs_at(c, b, ch * 8 + 8 + 2 * t4));
          uint32_t aw[3][4];
#pragma unroll
          for (int g = 0; g < 3; ++g) ldsm_x4(aw[g], smem_u32(wg[g]) + swz(arow, ch + ahalf, gh * 2));
#pragma unroll
          for (int nt = 0; nt < 2; ++nt) {
            // history row of level l = 8 nt + (lane & 7); levels without a
            // source (or beyond L) read the zero row
            const int l = nt * 8 + brow;
            const bool ok = l < L && t - (1ll << l) >= 0;
            const uint8_t* rowp = ok ? bhc[b] + (size_t)l * bstride
                                     : reinterpret_cast<const uint8_t*>(c.zrow);
            uint32_t bf[2];
            ldsm_x2(bf, smem_u32(rowp + (ch + bhalf) * 16));
            __nv_bfloat162 h0 = __hmax2(__hadd2(a_lo, *reinterpret_cast<__nv_bfloat162*>(&bf[0])), z2);
            __nv_bfloat162 h1 = __hmax2(__hadd2(a_hi, *reinterpret_cast<__nv_bfloat162*>(&bf[1])), z2);
            h0 = __hmul2(h0, h0);  // relu squared, rounded to bf16 as the reference's fused gates
            h1 = __hmul2(h1, h1);
            uint32_t hv[2] = {*reinterpret_cast<uint32_t*>(&h0), *reinterpret_cast<uint32_t*>(&h1)};
#pragma unroll
            for (int g = 0; g < 3; ++g) mma16816(acc[g][nt], aw[g], hv);
          }
        }
      }
      float acc[3][2][4];
#pragma unroll
      for (int g = 0; g < 3; ++g)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int e = 0; e < 4; ++e) acc[g][nt][e] = acc2[0][g][nt][e] + acc2[1][g][nt][e];
      // diagonal: level l = g4 sits in acc[..][0][0] when g4 == 2 t4 and in
      // acc[..][0][1] when g4 == 2 t4 + 1; level 8 + g4 likewise in [1][2] / [1][3]
      float* rb = red + ((size_t)warp * kMaxB + b) * 48;
#pragma unroll
      for (int g = 0; g < 3; ++g) {
        if (g4 == 2 * t4) {
          rb[g * 16 + g4] = acc[g][0][0];
          rb[g * 16 + g4 + 8] = acc[g][1][2];
        } else if (g4 == 2 * t4 + 1) {
          rb[g * 16 + g4] = acc[g][0][1];
          rb[g * 16 + g4 + 8] = acc[g][1][3];
        }
      }
    }
  }
  for (int b = 0; b < B + 3; ++b) chunk_release(c);
  csync();
  // sigmoid gates; transmit gate of position t into rg_hist
  for (int i = tid; i < B * L; i += kCons) {
    const int b = i / L, l = i - b * L;
    float pre[3];
#pragma unroll
    for (int g = 0; g < 3; ++g) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) s += red[((size_t)w * kMaxB + b) * 48 + g * 16 + l];
      pre[g] = s + s_bias[l * 3 + g];
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
#pragma unroll 1
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
    *reinterpret_cast<uint4*>(s_y + b * 64 + g * 8) = pack8(V);  // y is bf16, as the reference's
  }
  csync();
  // out-projection share on the tensor cores: x[b, n] += sum_c W_out[n, h*hd + c] y_h[b, c]
  // for this CTA's half of the rows n, added into both residual buffers.
  // A = 16-row tiles of the (swizzled) head block, B = y rows (hd = 64: 4 k-steps).
  uint32_t by[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int n = lane & 7, half = (lane >> 3) & 1;
    const __nv_bfloat16* row = n < B ? s_y + n * 64 + (2 * i + half) * 8 : c.zrow + (2 * i + half) * 8;
    ldsm_x2(by[i], smem_u32(row));
  }
  const Seg so = get_seg(c, li, PH_B, 2);
  const int upc = units_per_chunk(c, so);
  const int nbase = c.hpart * (d / kHeadParts);
  const int arow = (lane & 7) + ((lane >> 3) & 1) * 8, ahalf = lane >> 4;
  for (int cu = 0; cu < so.units; cu += upc) {
    const int ntile = min(upc, so.units - cu);
    const uint8_t* chunk = chunk_acquire(c);
    for (int mt = warp; mt < ntile; mt += kWarps) {
      const uint32_t tb = smem_u32(chunk) + (uint32_t)mt * 16 * hd * 2;
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        uint32_t a[4];
        ldsm_x4(a, tb + swz(arow, 2 * i + ahalf, hd * 2));
        mma16816(acc, a, by[i]);
      }
      const int n0 = nbase + (cu + mt) * 16 + g4;
      if (2 * t4 < B) {
        red_add_f32(c.p.x + (size_t)(2 * t4) * d + n0, acc[0]);
        red_add_f32(c.p.x_in + (size_t)(2 * t4) * d + n0, acc[0]);
        red_add_f32(c.p.x + (size_t)(2 * t4) * d + n0 + 8, acc[2]);
        red_add_f32(c.p.x_in + (size_t)(2 * t4) * d + n0 + 8, acc[2]);
      }
      if (2 * t4 + 1 < B) {
        red_add_f32(c.p.x + (size_t)(2 * t4 + 1) * d + n0, acc[1]);
        red_add_f32(c.p.x_in + (size_t)(2 * t4 + 1) * d + n0, acc[1]);
        red_add_f32(c.p.x + (size_t)(2 * t4 + 1) * d + n0 + 8, acc[3]);
        red_add_f32(c.p.x_in + (size_t)(2 * t4 + 1) * d + n0 + 8, acc[3]);
      }
    }
    chunk_release(c);
  }
  stamp(c, li, PH_B, 3);
  grid_arrive(c, li, PH_B);
}

// GEMV CTAs: split-window attention with last-arriver combine
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
__device__ void phase_o(Ctx& c, int li) {
  const int d = c.d;
  stamp(c, li, PH_O, 0);
  grid_wait(c, li, PH_B, c.B * c.H);
  stamp(c, li, PH_O, 1);
  stage_copy(c, static_cast<const __nv_bfloat16*>(c.p.y), d);
  stamp(c, li, PH_O, 2);
  const int ksw = d / 128;
  uint32_t bx[8][2];
  load_xfrags(c, ksw, bx);
  int u0, u1;
  split_range(d / 16, c.NG, c.cta, u0, u1);
  const Seg s = get_seg(c, li, PH_O, 0);
  float* x = c.p.x;
  float* xin = c.p.x_in;
  gemv_tiles(c, s, bx, ksw, [&](int u, int p, int b, float ve, float vo) {
    const size_t i = (size_t)b * d + (u0 + u) * 16 + 2 * p;
    const float2 old = __ldcg(reinterpret_cast<const float2*>(x + i));
    const float2 nx = make_float2(old.x + ve, old.y + vo);
    *reinterpret_cast<float2*>(x + i) = nx;
    *reinterpret_cast<float2*>(xin + i) = nx;
  });
  stamp(c, li, PH_O, 3);
  grid_arrive(c, li, PH_O);
}

// GEMV CTAs: the FFN slice, down projection added into x
__device__ void phase_c(Ctx& c, int li) {
  const dh_layer_params& lp = layer(c, li);
  const int d = c.d, B = c.B, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g4 = lane >> 2, t4 = lane & 3;
  stamp(c, li, PH_C, 0);
  const NormW nw = load_normw(c, static_cast<const __nv_bfloat16*>(lp.norm2));
  if (lp.kind == 0) grid_wait(c, li, PH_B, c.H * kHeadParts);
  else grid_wait(c, li, PH_O, c.NG);
  stamp(c, li, PH_C, 1);
  stage_norm(c, c.p.x_in, nw);
  stamp(c, li, PH_C, 2);
  const int ksw = d / 128;
  uint32_t bx[8][2];
  load_xfrags(c, ksw, bx);
  int t0, t1;
  split_range(c.ff / 8, c.NG, c.cta, t0, t1);
  const int jn = 8 * (t1 - t0);  // FFN columns of this CTA
  float* us = c.misc;            // [kMaxB][kMaxUpc] (u rounded to bf16)
  const Seg sgu = get_seg(c, li, PH_C, 0);
  gemv_tiles(c, sgu, bx, ksw, [&](int u, int p, int b, float gate, float up) {
    us[b * kMaxUpc + u * 8 + p] = bf2f(f2bf(gate / (1.0f + expf(-gate)) * up));
  });
  csync();
  // down projection on the tensor cores: D[b, n] = sum_j u[b, j] Wd[n, j0 + j]
  // with A = u (rows = lockstep rows) and B = 16-row tiles of Wd^T (one per
  // chunk, read transposed by ldmatrix); warp w takes n-tiles w, w + 8, ...
  const Seg sd = get_seg(c, li, PH_C, 1);
  float acc[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
  const int ntiles = d / 8;  // 8-column tiles of n
  for (int kt = 0; kt < sd.units; ++kt) {
    const uint8_t* chunk = chunk_acquire(c);
    const int kvalid = min(16, jn - kt * 16);
    uint32_t au[4] = {0u, 0u, 0u, 0u};
    if (g4 < B) {
      const int k0 = kt * 16 + 2 * t4;
      const float* ur = us + g4 * kMaxUpc;
      au[0] = k0 < jn ? pack2(ur[k0], ur[k0 + 1]) : 0u;
      au[2] = k0 + 8 < jn ? pack2(ur[k0 + 8], ur[k0 + 9]) : 0u;
    }
    const uint32_t base = smem_u32(chunk);
    const int krow = (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int nt = warp + kWarps * i;
      if (nt < ntiles) {
        uint32_t bw[2];
        ldsm_x2_t(bw, base + swz(krow, nt, d * 2));
        if (kvalid <= 8) bw[1] = 0u;  // rows past this CTA's columns hold stale data
        mma16816(acc[i], au, bw);     // only rows b < B (acc[.][0..1]) are kept
      }
    }
    chunk_release(c);
  }
  if (g4 < B && sd.units > 0) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int nt = warp + kWarps * i;
      if (nt < ntiles) red_add_v2(c.p.x + (size_t)g4 * d + nt * 8 + 2 * t4, acc[i][0], acc[i][1]);
    }
  }
  stamp(c, li, PH_C, 3);
  grid_arrive(c, li, PH_C);
}

__device__ void phase_n(Ctx& c) {
  const int d = c.d, nl = c.p.n_layers;
  stamp(c, nl, 0, 0);
  const NormW nw = load_normw(c, static_cast<const __nv_bfloat16*>(c.p.norm_out));
  grid_wait(c, nl - 1, PH_C, c.NG);
  stamp(c, nl, 0, 1);
  stage_norm(c, c.p.x, nw);
  stamp(c, nl, 0, 2);
  const int ksw = d / 128;
  uint32_t bx[8][2];
  load_xfrags(c, ksw, bx);
  int u0, u1;
  const int V = c.p.vocab;
  split_range((V + 15) / 16, c.G, c.cta, u0, u1);
  const Seg s = get_seg(c, nl, PH_N, 0);
  __nv_bfloat16* lg = static_cast<__nv_bfloat16*>(c.p.logits);
  gemv_tiles(c, s, bx, ksw, [&](int u, int p, int b, float ve, float vo) {
    const int n = (u0 + u) * 16 + 2 * p;
    if (n < V) lg[(size_t)b * V + n] = f2bf(ve);
    if (n + 1 < V) lg[(size_t)b * V + n + 1] = f2bf(vo);
  });
  stamp(c, nl, 0, 3);
}

// ------------------------------------------------------------------ kernel
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
  // ring slots, then the attention staging buffer, which head CTAs (never
  // in an attention phase) use as one more ring slot
  static_assert(2 * kKvPos * 64 * 2 == kSlotBytes, "the staging buffer doubles as a slot");
  c.nslots = c.head >= 0 ? kSlots + 1 : kSlots;
  c.slots = smem_raw;
  c.kv = reinterpret_cast<__nv_bfloat16*>(smem_raw + (size_t)kSlots * kSlotBytes);
  uint8_t* q = smem_raw + (size_t)(kSlots + 1) * kSlotBytes;
  c.xs = reinterpret_cast<__nv_bfloat16*>(q);
  q += (size_t)kMaxB * kMaxD * 2;
  c.zrow = reinterpret_cast<__nv_bfloat16*>(q);
  q += (size_t)kMaxD * 2;
  c.red = reinterpret_cast<float*>(q);
  q += (size_t)2 * kWarps * 16 * 8 * 4;
  c.misc = reinterpret_cast<float*>(q);
  q += (size_t)kMisc * 4;
  c.full = reinterpret_cast<uint64_t*>(q);
  c.empty = c.full + kSlots + 1;
  c.abort = reinterpret_cast<volatile int*>(c.empty + kSlots + 1);
  c.prod = reinterpret_cast<Prod*>(const_cast<int*>(reinterpret_cast<volatile int*>(c.abort)) + 4);
  c.acq = 0;
  c.rel = 0;
  c.t = __ldcg(p.t_buf);
  c.gen = __ldcg(p.barrier);
  if (c.t < 0 || c.t >= p.max_len) {  // no position left: nothing is written
    if (c.cta == 0 && threadIdx.x == 0) atomicExch(p.status, DH_ERR_ARG);
    return;
  }
  {  // the layer table, read once into shared memory; the zero row
    dh_layer_params* lay = reinterpret_cast<dh_layer_params*>(
        reinterpret_cast<uint8_t*>(c.prod) + ((sizeof(Prod) + 15) / 16) * 16);
    const unsigned long long* src = reinterpret_cast<const unsigned long long*>(p.layers);
    unsigned long long* dst = reinterpret_cast<unsigned long long*>(lay);
    const int words = p.n_layers * (int)(sizeof(dh_layer_params) / 8);
    for (int i = threadIdx.x; i < words; i += kThreads) dst[i] = src[i];
    for (int i = threadIdx.x; i < kMaxD / 8; i += kThreads)
      reinterpret_cast<uint4*>(c.zrow)[i] = make_uint4(0, 0, 0, 0);
    c.lay = lay;
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < c.nslots; ++s) {
      mbar_init(&c.full[s], 1);
      mbar_init(&c.empty[s], kWarps);
    }
    *c.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    Prod* pr = c.prod;
    pr->lay = c.lay;
    pr->lm_head = p.lm_head;
    pr->vocab = p.vocab;
    pr->max_len = p.max_len;
    pr->n_layers = p.n_layers;
    pr->G = c.G; pr->cta = c.cta; pr->NG = c.NG; pr->head = c.head; pr->hpart = c.hpart;
    pr->B = c.B; pr->d = c.d; pr->gh = c.gh; pr->L = c.L; pr->H = c.H; pr->hd = c.hd;
    pr->ff = c.ff; pr->nslots = c.nslots; pr->t = c.t;
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
      phase_a(c, li);
      if (tree) {
        phase_c(c, li);
      } else {
        phase_b_attn(c, li);
        phase_o(c, li);
        phase_c(c, li);
      }
    } else if (tree) {
      phase_b_tree(c, li);
    }
  }
  phase_n(c);
  cp_async_wait_all();
  stamp(c, p.n_layers, 1, 1);
  if (c.cta == 0 && threadIdx.x == 0) {
    p.t_buf[0] = c.t + 1;
    atomicAdd(p.barrier, 1ull);
  }
}

size_t step_smem() {
  return (size_t)(kSlots + 1) * kSlotBytes + (size_t)kMaxB * kMaxD * 2 + (size_t)kMaxD * 2 +
         (size_t)2 * kWarps * 16 * 8 * 4 + (size_t)kMisc * 4 + (size_t)2 * (kSlots + 1) * 8 + 16 +
         ((sizeof(Prod) + 15) / 16) * 16 + (size_t)kMaxLayers * sizeof(dh_layer_params);
}

int launch_step(const dh_step_params& p, cudaStream_t st) {
  const size_t smem = step_smem();
  DH_REQUIRE(smem <= 227 * 1024, DH_ERR_SHAPE, "dh_decode_step: %zu bytes of shared memory", smem);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    configured_dev = dev;
  }
  int per_sm = 0;
  const cudaError_t occ =
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel, kThreads, smem);
  if (per_sm < 1) {
    cudaFuncAttributes fa{};
    cudaFuncGetAttributes(&fa, step_kernel);
    return set_error(DH_ERR_SHAPE,
                     "dh_decode_step: kernel does not fit on an SM (%s; %d regs, %zu B smem "
                     "requested, max dynamic %d, max threads %d)",
                     cudaGetErrorString(occ), fa.numRegs, smem, fa.maxDynamicSharedSizeBytes,
                     fa.maxThreadsPerBlock);
  }
  const int G = sm_count();
  const int NG = G - p.H * kHeadParts;
  DH_REQUIRE(NG >= 16, DH_ERR_SHAPE, "dh_decode_step: %d SMs leave too few GEMV CTAs", G);
  DH_REQUIRE(8 * ((p.ff / 8 + NG - 1) / NG) <= kMaxUpc, DH_ERR_SHAPE,
             "dh_decode_step: FFN width %d too large for %d CTAs", p.ff, NG);
  {  // the attention scores of one item live in the per-phase scratch
    const int span = (p.window > 0 && p.window < p.max_len) ? p.window : p.max_len;
    int ns = NG / (p.batch * p.H);
    ns = ns < 1 ? 1 : (ns < p.nsplit ? ns : p.nsplit);
    const int chunk = (span + ns - 1) / ns;
    DH_REQUIRE(chunk + 64 + 8 + kWarps * 64 + 4 <= kMisc - kMaxB, DH_ERR_SHAPE,
               "dh_decode_step: %d window positions per attention item exceed the scratch", chunk);
  }
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
  if (cudaLaunchKernelEx(&cfg, step_kernel, p, wait_limit()) != cudaSuccess)
    return check_launch("step_kernel");
  return DH_OK;
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_decode_step(const dh_step_params* params, void* stream) {
  DH_REQUIRE(params, DH_ERR_ARG, "dh_decode_step: null params");
  const dh_step_params& p = *params;
  DH_REQUIRE(p.layers && p.tokens && p.t_buf && p.emb && p.lm_head && p.norm_out && p.logits &&
                 p.x && p.x_in && p.a && p.v0 && p.y && p.q && p.part && p.counters && p.barrier &&
                 p.status,
             DH_ERR_ARG, "dh_decode_step: null pointer in params");
  DH_REQUIRE(p.batch >= 1 && p.batch <= kMaxB, DH_ERR_SHAPE,
             "dh_decode_step: batch %d not in [1,%d]", p.batch, kMaxB);
  DH_REQUIRE(p.hd == 64 && p.d == p.H * p.hd && p.d % 128 == 0 && p.d <= kMaxD && p.ff % 16 == 0 &&
                 p.L >= 1 && p.L <= kLmax && p.L * (2 * p.d + 16) <= kSlotBytes && p.nsplit >= 1 &&
                 p.n_layers >= 1 && p.n_layers <= kMaxLayers,
             DH_ERR_SHAPE, "dh_decode_step: unsupported shape (d=%d H=%d hd=%d ff=%d L=%d layers=%d)",
             p.d, p.H, p.hd, p.ff, p.L, p.n_layers);
  return launch_step(p, reinterpret_cast<cudaStream_t>(stream));
}
