// Whole decode step as ONE persistent cooperative kernel (one CTA per SM).
//
// A step is a fixed sequence of phases (embedding; per block: input
// projection, mixer or attention, output projection + residual, FFN input,
// FFN down + residual; logits).  Every weight matrix of a phase is split into
// contiguous row ranges, one per CTA, so each weight byte crosses HBM once per
// step.  Weights never depend on activations: each CTA runs a weight stream —
// its slices of all phases, in phase order, cut into chunks and copied by
// bulk async copies (cp.async.bulk) into a ring of shared-memory slots — that
// runs ahead of the grid barriers.  After a barrier a phase only reads the
// (small) activation vector of the lockstep batch from L2 and computes from
// shared memory.
//
// The tree block's gates + level recurrence keep the structure of the
// per-op kernel (fused_step.py:26-88 semantics): CTAs own (level, head)
// items, and the last CTA to finish a head runs that head's recurrence.
//
// Grid barrier: a monotonically increasing 64-bit arrival counter; every
// wait is bounded and a timeout sets *status, after which the kernel keeps
// going without waiting (wrong data, but it always terminates).
#include <math.h>

#include "common.cuh"

namespace dh {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr float kEps = 1.1920928955078125e-07f;  // torch RMSNorm eps=None in fp32
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr int kSlots = 3;          // weight-stream slots in shared memory
constexpr int kSlotBytes = 40960;  // bytes per slot (a chunk is whole units)

// ------------------------------------------------------------------ ctx
struct Ctx {
  const dh_step_params& p;  // the kernel's __grid_constant__ parameter
  int G, cta;
  unsigned long long base;  // barrier counter value at launch
  int nbar;                 // barriers passed so far in this launch
  long long t;              // position of this step
  __nv_bfloat16* xs;        // staged input activations [batch][K]
  float* red;               // small CTA-wide scratch
  uint8_t* slots;           // weight-stream slots, kSlots x kSlotBytes
  uint64_t* full;           // one mbarrier per slot
  int* cursor;              // producer state in shared memory: phase, next unit, issued
  int consumed;             // chunks consumed so far (same on every thread)
};

__device__ __forceinline__ void grid_sync(Ctx& c) {
  c.nbar += 1;
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long target = c.base + (unsigned long long)c.nbar * c.G;
    __threadfence();
    atomicAdd(c.p.barrier, 1ull);
    unsigned long long v = 0;
    uint32_t it = 0;
    while (true) {
      asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(c.p.barrier) : "memory");
      if (v >= target) break;
      if (++it > kSpinLimit) {
        atomicExch(c.p.status, DH_ERR_TIMEOUT);
        break;
      }
      __nanosleep(32);
    }
    __threadfence();
  }
  __syncthreads();
}

__device__ __forceinline__ void split_range(int n, int G, int c, int& a, int& b) {
  a = (int)((long long)n * c / G);
  b = (int)((long long)n * (c + 1) / G);
}

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

// ------------------------------------------------------------------ input staging
// xs[b][k] = bf16(x[b][k] * rsqrt(mean(x[b]^2) + eps) * w[k]) for the lockstep rows.
// The rows are spread over all threads (one L2 round trip), squares are
// summed per row with shared-memory atomics, and the values stay in registers.
constexpr int kStageV = 16;  // float4 per thread: batch * K <= 16 * 1024
template <int NV>  // float4 per thread, NV * 1024 >= batch * K
__device__ __forceinline__ void stage_norm(Ctx& c, const float* x, const __nv_bfloat16* w, int K) {
  const int B = c.p.batch, k4 = K / 4, n4 = B * k4;
  float* ssum = c.red;  // [16]
  if (threadIdx.x < 16) ssum[threadIdx.x] = 0.f;
  __syncthreads();
  float4 v[NV];
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * kThreads;
    float sq = 0.f;
    if (i < n4) {
      v[j] = __ldcg(reinterpret_cast<const float4*>(x) + i);
      sq = v[j].x * v[j].x + v[j].y * v[j].y + v[j].z * v[j].z + v[j].w * v[j].w;
    }
    if ((k4 & 31) == 0) {  // a warp's 32 float4 lie in one row: reduce, one atomic
      sq = warp_sum(sq);
      if ((threadIdx.x & 31) == 0 && i < n4) atomicAdd(&ssum[i / k4], sq);
    } else if (i < n4) {
      atomicAdd(&ssum[i / k4], sq);
    }
  }
  __syncthreads();
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = threadIdx.x + j * kThreads;
    if (i < n4) {
      const int b = i / k4, k = (i - b * k4) * 4;
      const float r = rsqrtf(ssum[b] / (float)K + kEps);
      const uint2 wv = *reinterpret_cast<const uint2*>(w + k);
      const float2 w01 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.x));
      const float2 w23 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&wv.y));
      uint2 pk;
      pk.x = pack2(v[j].x * r * w01.x, v[j].y * r * w01.y);
      pk.y = pack2(v[j].z * r * w23.x, v[j].w * r * w23.y);
      *reinterpret_cast<uint2*>(c.xs + (size_t)b * K + k) = pk;
    }
  }
  __syncthreads();
}

// xs = src (bf16, batch rows of K)
__device__ __forceinline__ void stage_copy(Ctx& c, const __nv_bfloat16* src, int K) {
  const int n = c.p.batch * K / 8;
  const uint4* s4 = reinterpret_cast<const uint4*>(src);
  uint4* d4 = reinterpret_cast<uint4*>(c.xs);
  for (int i0 = threadIdx.x; i0 < n; i0 += 8 * kThreads) {  // 8 loads in flight per thread
    uint4 v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j * kThreads;
      if (i < n) v[j] = __ldcg(s4 + i);
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int i = i0 + j * kThreads;
      if (i < n) d4[i] = v[j];
    }
  }
  __syncthreads();
}

// ------------------------------------------------------------------ weight stream
// Phase pi (0 .. 5*n_layers) of a step: per block 0 = input projection, 1 =
// mixer gates (tree) / attention (no weights), 2 = output projection, 3 = FFN
// input (gate/up pairs), 4 = FFN down; the last phase is the logits.  A unit
// is the smallest contiguous weight piece one warp consumes.
struct PhaseW {
  const uint8_t* base;
  int unit_bytes, units;
  size_t total;  // bytes of the whole matrix (the last unit may be short)
};

__device__ PhaseW phase_weights(const dh_step_params& p, int pi) {
  const int d = p.d, nl = p.n_layers;
  PhaseW w{nullptr, 1, 0, 0};
  if (pi >= 5 * nl) {
    w.base = static_cast<const uint8_t*>(p.emb);
    w.unit_bytes = 4 * d;
    w.units = (p.vocab + 1) / 2;
    w.total = (size_t)p.vocab * d * 2;
    return w;
  }
  const dh_layer_params& lp = p.layers[pi / 5];
  switch (pi % 5) {
    case 0: w.base = static_cast<const uint8_t*>(lp.w_in3); w.unit_bytes = 4 * d; w.units = 3 * d / 2; break;
    case 1:
      if (lp.kind == 0) {
        w.base = static_cast<const uint8_t*>(lp.w_gates);
        w.unit_bytes = 6 * d;
        w.units = p.L * p.H;
      }
      break;
    case 2: w.base = static_cast<const uint8_t*>(lp.w_out); w.unit_bytes = 4 * d; w.units = d / 2; break;
    case 3: w.base = static_cast<const uint8_t*>(lp.w_gu); w.unit_bytes = 4 * d; w.units = p.ff; break;
    default: w.base = static_cast<const uint8_t*>(lp.w_down); w.unit_bytes = 4 * p.ff; w.units = d / 2; break;
  }
  w.total = (size_t)w.units * w.unit_bytes;
  return w;
}

__device__ __forceinline__ int units_per_chunk(int unit_bytes) {
  int n = kSlotBytes / unit_bytes;
  if (n >= kWarps) n -= n % kWarps;  // whole rounds of warps
  return n < 1 ? 1 : n;
}

__device__ __forceinline__ void bulk_copy_g2s(void* dst, const void* src, uint32_t bytes,
                                              uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Issue the next chunk of this CTA's weight stream (called by thread 0 only,
// each time a slot is free).  Returns false when the stream is exhausted.
__device__ bool issue_next(Ctx& c) {
  int pi = c.cursor[0], u = c.cursor[1];
  const int np = 5 * c.p.n_layers + 1;
  while (pi < np) {
    const PhaseW w = phase_weights(c.p, pi);
    int u0, u1;
    split_range(w.units, c.G, c.cta, u0, u1);
    if (u < u0) u = u0;
    if (u < u1) {
      const int n = min(units_per_chunk(w.unit_bytes), u1 - u);
      const size_t off = (size_t)u * w.unit_bytes;
      size_t bytes = (size_t)n * w.unit_bytes;
      if (off + bytes > w.total) bytes = w.total - off;
      const int slot = c.cursor[2] % kSlots;
      mbar_arrive_expect_tx(&c.full[slot], (uint32_t)bytes);
      bulk_copy_g2s(c.slots + (size_t)slot * kSlotBytes, w.base + off, (uint32_t)bytes,
                    &c.full[slot]);
      c.cursor[0] = pi;
      c.cursor[1] = u + n;
      c.cursor[2] += 1;
      return true;
    }
    ++pi;
    u = 0;
  }
  c.cursor[0] = pi;
  c.cursor[1] = 0;
  return false;
}

// Consumer side: wait for the next chunk; returns its shared-memory base.
__device__ __forceinline__ const uint8_t* chunk_wait(Ctx& c) {
  const int slot = c.consumed % kSlots;
  mbar_wait(&c.full[slot], (uint32_t)((c.consumed / kSlots) & 1), c.p.status, 1u << 22);
  return c.slots + (size_t)slot * kSlotBytes;
}

// All threads are done with the current chunk: refill its slot.
__device__ __forceinline__ void chunk_release(Ctx& c) {
  __syncthreads();
  if (threadIdx.x == 0) issue_next(c);
  c.consumed += 1;
}

// ------------------------------------------------------------------ GEMV phases
enum { E_MIXIN = 0, E_QKV = 1, E_RESID = 2, E_FFNIN = 3, E_LOGITS = 4 };

struct GemvPhase {
  int epi;
  int K;                        // input width
  int N;                        // output rows of the weight (RESID / LOGITS)
  const __nv_bfloat16* norm_w;  // staging: RMSNorm of x with this weight, or
  const __nv_bfloat16* src;     // staging: copy this bf16 (batch, K) buffer
  float* x;                     // residual stream (RESID)
  __nv_bfloat16 *o0, *o1, *o2;  // outputs (see store_unit)
};

// value v of output row `row` (0/1) of unit u for batch row b; `other` is the
// partner row's value (SwiGLU and RoPE pairs)
__device__ __forceinline__ void store_unit(const Ctx& c, const GemvPhase& g, int u, int b, int row,
                                           float v, float other, bool has1) {
  const int d = c.p.d;
  switch (g.epi) {
    case E_MIXIN: {  // [W_in; W1x; W1s] -> v0, A, B_hist[:, t]
      const int n = 2 * u + row, seg = n / d, col = n - seg * d;
      if (seg == 0) g.o0[(size_t)b * d + col] = f2bf(v);
      else if (seg == 1) g.o1[(size_t)b * d + col] = f2bf(v);
      else g.o2[((size_t)b * c.p.max_len + c.t) * d + col] = f2bf(v);
      break;
    }
    case E_QKV: {  // [Wq; Wk; Wv], RoPE at t on q and k; k, v into the caches
      const int n = 2 * u + row, seg = n / d, col = n - seg * d, hd = c.p.hd;
      float out = v;
      if (seg < 2) {
        const int j = (col % hd) >> 1;
        const float cs = c.p.rope_cos[c.t * (hd / 2) + j], sn = c.p.rope_sin[c.t * (hd / 2) + j];
        const float x1 = row == 0 ? v : other, x2 = row == 0 ? other : v;
        out = row == 0 ? (x1 * cs - x2 * sn) : (x1 * sn + x2 * cs);
      }
      if (seg == 0) g.o0[(size_t)b * d + col] = f2bf(out);
      else if (seg == 1) g.o1[((size_t)b * c.p.max_len + c.t) * d + col] = f2bf(out);
      else g.o2[((size_t)b * c.p.max_len + c.t) * d + col] = f2bf(out);
      break;
    }
    case E_RESID: {  // x += W . input (this CTA owns these rows)
      float* p = g.x + (size_t)b * g.N + 2 * u + row;
      *p = __ldcg(p) + v;
      break;
    }
    case E_FFNIN:  // unit j = (gate_j, up_j): u_j = silu(g) * up
      if (row == 0) g.o0[(size_t)b * c.p.ff + u] = f2bf(v / (1.0f + expf(-v)) * other);
      break;
    default:  // logits
      if (row == 1 && !has1) break;
      g.o0[(size_t)b * g.N + 2 * u + row] = f2bf(v);
  }
}

template <int MAXB>
__device__ __forceinline__ void dot_pair_smem(const __nv_bfloat16* r0, const __nv_bfloat16* r1,
                                              int K, const __nv_bfloat16* xs, int batch,
                                              float (&acc)[2 * MAXB]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int i = 0; i < 2 * MAXB; ++i) acc[i] = 0.f;
  for (int k = lane * 8; k < K; k += 256) {
    float fa[8], fb[8];
    unpack8(*reinterpret_cast<const uint4*>(r0 + k), fa);
    unpack8(*reinterpret_cast<const uint4*>(r1 + k), fb);
#pragma unroll
    for (int b = 0; b < MAXB; ++b) {
      if (b < batch) {
        float fx[8];
        unpack8(*reinterpret_cast<const uint4*>(xs + (size_t)b * K + k), fx);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[b] = fmaf(fa[j], fx[j], acc[b]);
          acc[MAXB + b] = fmaf(fb[j], fx[j], acc[MAXB + b]);
        }
      }
    }
  }
}

// grid barrier, stage the input, then consume this CTA's chunks of phase pi
template <int MAXB>
__device__ __noinline__ void gemv_phase(Ctx& c, int pi, const GemvPhase& g) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const PhaseW w = phase_weights(c.p, pi);
  int u0, u1;
  split_range(w.units, c.G, c.cta, u0, u1);
  grid_sync(c);
  if (g.norm_w) stage_norm<MAXB>(c, c.p.x, g.norm_w, g.K);
  else stage_copy(c, g.src, g.K);
  const int upc = units_per_chunk(w.unit_bytes);
  for (int cu0 = u0; cu0 < u1; cu0 += upc) {
    const int cu1 = min(cu0 + upc, u1);
    const uint8_t* chunk = chunk_wait(c);
    for (int u = cu0 + warp; u < cu1; u += kWarps) {
      const __nv_bfloat16* r0 =
          reinterpret_cast<const __nv_bfloat16*>(chunk + (size_t)(u - cu0) * w.unit_bytes);
      const bool has1 = (size_t)(u + 1) * w.unit_bytes <= w.total;
      const __nv_bfloat16* r1 = has1 ? r0 + g.K : r0;
      float acc[2 * MAXB];
      dot_pair_smem<MAXB>(r0, r1, g.K, c.xs, c.p.batch, acc);
      const float r = transpose_reduce<2 * MAXB>(acc);
      const float other = __shfl_xor_sync(0xffffffffu, r, MAXB);
      const int b = lane % MAXB, row = (lane / MAXB) & 1;
      if (lane < 2 * MAXB && b < c.p.batch) store_unit(c, g, u, b, row, r, other, has1);
    }
    chunk_release(c);
  }
}

// ------------------------------------------------------------------ tree phase
// Items (level, head); the two 128-thread halves of the CTA take alternate
// items of each chunk.  Each item: the three gate readouts of every lockstep
// row (fused_step.py:26-59), then the last CTA to finish a head runs that
// head's level recurrence (fused_step.py:62-88, fp32 state).
template <int MAXB>
__device__ __noinline__ void tree_phase(Ctx& c, int pi, const dh_layer_params& lp) {
  const int L = c.p.L, H = c.p.H, hd = c.p.hd, gh = c.p.d, d = H * hd, B = c.p.batch;
  const int S = (1 << (L + 1)) - 2;
  const int half = threadIdx.x >> 7, gt = threadIdx.x & 127, hw = gt >> 5, lane = threadIdx.x & 31;
  const PhaseW w = phase_weights(c.p, pi);
  int i0, i1;
  split_range(w.units, c.G, c.cta, i0, i1);
  const __nv_bfloat16* a_in = static_cast<const __nv_bfloat16*>(c.p.a);
  const __nv_bfloat16* bh = static_cast<const __nv_bfloat16*>(lp.b_hist);
  __nv_bfloat16* rg = static_cast<__nv_bfloat16*>(lp.rg_hist);
  __nv_bfloat16* ring = static_cast<__nv_bfloat16*>(lp.v_ring);
  const __nv_bfloat16* v0 = static_cast<const __nv_bfloat16*>(c.p.v0);
  __nv_bfloat16* y = static_cast<__nv_bfloat16*>(c.p.y);
  float* red = c.red + 16 + half * (4 * 3 * 16 + 8);  // [4 warps][3*16] + flag
  int* flag = reinterpret_cast<int*>(red + 4 * 3 * 16);
  const long long t = c.t;
  grid_sync(c);
  const int upc = units_per_chunk(w.unit_bytes);
  for (int cu0 = i0; cu0 < i1; cu0 += upc) {
    const int cu1 = min(cu0 + upc, i1);
    const uint8_t* chunk = chunk_wait(c);
    for (int item = cu0 + half; item < cu1; item += 2) {
      const int l = item / H, h = item - l * H;
      const long long src = t - (1ll << l);
      const bool ok = src >= 0;
      const long long srcc = ok ? src : 0;
      const __nv_bfloat16* wi =
          reinterpret_cast<const __nv_bfloat16*>(chunk + (size_t)(item - cu0) * w.unit_bytes);
      float acc[MAXB][3];
#pragma unroll
      for (int b = 0; b < MAXB; ++b) acc[b][0] = acc[b][1] = acc[b][2] = 0.f;
      for (int k = gt * 8; k < gh; k += 1024) {
        float fw[3][8];
#pragma unroll
        for (int g = 0; g < 3; ++g) unpack8(*reinterpret_cast<const uint4*>(wi + (size_t)g * gh + k), fw[g]);
#pragma unroll
        for (int b = 0; b < MAXB; ++b) {
          if (b < B) {
            float fa[8], fs[8];
            unpack8(__ldcg(reinterpret_cast<const uint4*>(a_in + (size_t)b * gh + k)), fa);
            if (ok) {
              unpack8(__ldcg(reinterpret_cast<const uint4*>(bh + ((size_t)b * c.p.max_len + srcc) * gh + k)), fs);
            } else {
#pragma unroll
              for (int j = 0; j < 8; ++j) fs[j] = 0.f;
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              float hv = fmaxf(fa[j] + fs[j], 0.f);
              hv *= hv;  // relu squared
              acc[b][0] = fmaf(fw[0][j], hv, acc[b][0]);
              acc[b][1] = fmaf(fw[1][j], hv, acc[b][1]);
              acc[b][2] = fmaf(fw[2][j], hv, acc[b][2]);
            }
          }
        }
      }
#pragma unroll
      for (int b = 0; b < MAXB; ++b) {
#pragma unroll
        for (int g = 0; g < 3; ++g) {
          const float v = warp_sum(acc[b][g]);
          if (lane == 0 && b < B) red[hw * 48 + b * 3 + g] = v;
        }
      }
      asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
      if (gt < B) {
        const int b = gt;
        float pre[3];
#pragma unroll
        for (int g = 0; g < 3; ++g)
          pre[g] = red[b * 3 + g] + red[48 + b * 3 + g] + red[96 + b * 3 + g] + red[144 + b * 3 + g];
        const float* bg = lp.b_gates + (size_t)item * 3;
        const float okf = ok ? 1.f : 0.f;
        c.p.ig[((size_t)b * L + l) * H + h] = sigmoidf_(pre[0] + bg[0]) * okf;
        c.p.fg[((size_t)b * L + l) * H + h] = sigmoidf_(pre[1] + bg[1]) * okf + (1.f - okf);
        rg[(((size_t)b * c.p.max_len + t) * L + l) * H + h] = f2bf(sigmoidf_(pre[2] + bg[2]));
        __threadfence();
      }
      asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
      if (gt == 0) *flag = (atomicAdd(&c.p.counters[h], 1) == L - 1);
      asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
      if (*flag) {
        __threadfence();
        const int groups = hd / 8;
        if (gt < B * groups) {
          const int b = gt / groups;
          const int c0 = h * hd + (gt - b * groups) * 8;
          __nv_bfloat16* ringb = ring + (size_t)b * S * d;
          uint4 vsrc[16];
          float coef[16], fgv[16];
#pragma unroll
          for (int lv = 0; lv < 16; ++lv) {
            if (lv < L) {
              const long long s = t - (1ll << lv);
              fgv[lv] = __ldcg(c.p.fg + ((size_t)b * L + lv) * H + h);
              coef[lv] = 0.f;
              vsrc[lv] = make_uint4(0, 0, 0, 0);
              if (s >= 0) {
                const float igv = __ldcg(c.p.ig + ((size_t)b * L + lv) * H + h);
                const float rgv = bf2f(rg[(((size_t)b * c.p.max_len + s) * L + lv) * H + h]);
                coef[lv] = igv * rgv;
                const long long slot = ((2ll << lv) - 2) + (s & ((2ll << lv) - 1));
                vsrc[lv] = __ldcg(reinterpret_cast<const uint4*>(ringb + (size_t)slot * d + c0));
              }
            }
          }
          float V[8];
          const uint4 v0v = __ldcg(reinterpret_cast<const uint4*>(v0 + (size_t)b * d + c0));
          unpack8(v0v, V);
          *reinterpret_cast<uint4*>(ringb + (size_t)(t & 1) * d + c0) = v0v;
#pragma unroll
          for (int lv = 0; lv < 16; ++lv) {
            if (lv < L) {
              float vs[8];
              unpack8(vsrc[lv], vs);
#pragma unroll
              for (int j = 0; j < 8; ++j) V[j] = fgv[lv] * V[j] + coef[lv] * vs[j];
              if (lv + 1 < L) {
                const long long slot = ((2ll << (lv + 1)) - 2) + (t & ((2ll << (lv + 1)) - 1));
                *reinterpret_cast<uint4*>(ringb + (size_t)slot * d + c0) = pack8(V);
              }
            }
          }
          *reinterpret_cast<uint4*>(y + (size_t)b * d + c0) = pack8(V);
        }
        if (gt == 0) c.p.counters[h] = 0;
      }
      asm volatile("bar.sync %0, 128;" ::"r"(1 + half) : "memory");
    }
    chunk_release(c);
  }
}

// ------------------------------------------------------------------ attention phase
// Items (row, head, split): each CTA attends its chunk of the window with the
// whole block, writes a partial (max, sum, acc[hd]); the last split of a
// (row, head) combines the partials into y (decoding.py:260-264, 427-433).
__device__ __noinline__ void attn_phase(Ctx& c, const dh_layer_params& lp, float* sc) {
  constexpr int HD = 64;
  const int H = c.p.H, d = H * HD, B = c.p.batch, ns = c.p.nsplit;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const long long t = c.t;
  const long long lo = c.p.window > 0 ? (t + 1 - c.p.window > 0 ? t + 1 - c.p.window : 0) : 0;
  const long long n = t + 1 - lo;
  const long long chunk = (n + ns - 1) / ns;
  int i0, i1;
  split_range(B * H * ns, c.G, c.cta, i0, i1);
  grid_sync(c);
  const __nv_bfloat16* q = static_cast<const __nv_bfloat16*>(c.p.q);
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(lp.k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(lp.v_cache);
  float* sq = c.red + 512;         // [64]
  float* sred = c.red + 576;       // [8]
  float* sacc = c.red + 592;       // [8][64]
  int* flag = reinterpret_cast<int*>(c.red + 1104);
  const float scale = rsqrtf((float)HD);
  for (int item = i0; item < i1; ++item) {
    const int b = item / (H * ns), h = (item / ns) % H, split = item % ns;
    const long long s0 = lo + split * chunk;
    long long s1 = s0 + chunk;
    if (s1 > t + 1) s1 = t + 1;
    const int cnt = s1 > s0 ? (int)(s1 - s0) : 0;
    if (tid < HD) sq[tid] = bf2f(__ldcg(q + (size_t)b * d + h * HD + tid));
    __syncthreads();
    float mloc = -INFINITY;
#pragma unroll 2
    for (int i = tid; i < cnt; i += kThreads) {
      const uint4* kr = reinterpret_cast<const uint4*>(kc + ((size_t)b * c.p.max_len + s0 + i) * d + h * HD);
      float s = 0.f;
#pragma unroll
      for (int j = 0; j < HD / 8; ++j) {
        float f[8];
        unpack8(__ldcg(kr + j), f);
#pragma unroll
        for (int e = 0; e < 8; ++e) s = fmaf(f[e], sq[j * 8 + e], s);
      }
      s *= scale;
      sc[i] = s;
      mloc = fmaxf(mloc, s);
    }
    mloc = warp_max(mloc);
    if (lane == 0) sred[warp] = mloc;
    __syncthreads();
    float M = sred[0];
    for (int w = 1; w < kWarps; ++w) M = fmaxf(M, sred[w]);
    __syncthreads();
    float lsum = 0.f;
    for (int i = tid; i < cnt; i += kThreads) {
      const float e = expf(sc[i] - M);
      sc[i] = e;
      lsum += e;
    }
    lsum = warp_sum(lsum);
    if (lane == 0) sred[warp] = lsum;
    __syncthreads();
    float Ls = 0.f;
    for (int w = 0; w < kWarps; ++w) Ls += sred[w];
    // P V: 32 lanes x 2 channels, 8 warps over positions
    const int c2 = lane * 2;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll 8
    for (int i = warp; i < cnt; i += kWarps) {
      const __nv_bfloat162 vv = __ldcg(reinterpret_cast<const __nv_bfloat162*>(
          vc + ((size_t)b * c.p.max_len + s0 + i) * d + h * HD + c2));
      const float2 f = __bfloat1622float2(vv);
      a0 = fmaf(sc[i], f.x, a0);
      a1 = fmaf(sc[i], f.y, a1);
    }
    sacc[warp * HD + c2] = a0;
    sacc[warp * HD + c2 + 1] = a1;
    __syncthreads();
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
    __syncthreads();
    if (tid == 0) *flag = (atomicAdd(&c.p.counters[H + b * H + h], 1) == ns - 1);
    __syncthreads();
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
        static_cast<__nv_bfloat16*>(c.p.y)[(size_t)b * d + h * HD + tid] =
            f2bf(den > 0.f ? num / den : 0.f);
      }
      if (tid == 0) c.p.counters[H + b * H + h] = 0;
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------------ kernel
template <int MAXB>
__global__ void __launch_bounds__(kThreads, 1)
    step_kernel(const __grid_constant__ dh_step_params p, int xs_elems) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  Ctx c{p};
  c.G = gridDim.x;
  c.cta = blockIdx.x;
  c.nbar = 0;
  c.consumed = 0;
  c.slots = smem_raw;                                              // kSlots x kSlotBytes
  c.xs = reinterpret_cast<__nv_bfloat16*>(smem_raw + kSlots * kSlotBytes);
  c.red = reinterpret_cast<float*>(smem_raw + kSlots * kSlotBytes + (size_t)xs_elems * 2);
  float* sc = c.red + 1280;                                        // attention scores
  c.full = reinterpret_cast<uint64_t*>(c.red + 1272);              // 3 mbarriers (8-aligned)
  c.cursor = reinterpret_cast<int*>(c.red + 1266);
  const int nbar_total = 5 * p.n_layers + 1;
  c.t = __ldcg(p.t_buf);
  const unsigned long long gen = __ldcg(p.barrier + 1);
  c.base = gen * (unsigned long long)nbar_total * c.G;
  const int B = p.batch, d = p.d;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) mbar_init(&c.full[s], 1);
    fence_barrier_init();
    c.cursor[0] = 0;
    c.cursor[1] = 0;
    c.cursor[2] = 0;
    for (int s = 0; s < kSlots; ++s)
      if (!issue_next(c)) break;
  }
  __syncthreads();
  // embedding: x[b, :] = E[token[b], :] (this CTA's share of the 16-byte chunks)
  {
    int a, b;
    split_range(B * d / 8, c.G, c.cta, a, b);
    const __nv_bfloat16* emb = static_cast<const __nv_bfloat16*>(p.emb);
    for (int i = a + threadIdx.x; i < b; i += kThreads) {
      const int row = i / (d / 8), col = (i - row * (d / 8)) * 8;
      long long tok = p.tokens[row];
      if (tok < 0 || tok >= p.vocab) {
        atomicExch(p.status, 1);
        tok = tok < 0 ? 0 : p.vocab - 1;
      }
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(emb + (size_t)tok * d + col), f);
      float4* xo = reinterpret_cast<float4*>(p.x + (size_t)row * d + col);
      xo[0] = make_float4(f[0], f[1], f[2], f[3]);
      xo[1] = make_float4(f[4], f[5], f[6], f[7]);
    }
  }
  for (int li = 0; li < p.n_layers; ++li) {
    const dh_layer_params& lp = p.layers[li];
    const int pi = 5 * li;
    GemvPhase g{};
    g.K = d;
    g.norm_w = static_cast<const __nv_bfloat16*>(lp.norm1);
    if (lp.kind == 0) {
      g.epi = E_MIXIN;
      g.o0 = static_cast<__nv_bfloat16*>(p.v0);
      g.o1 = static_cast<__nv_bfloat16*>(p.a);
      g.o2 = static_cast<__nv_bfloat16*>(lp.b_hist);
      gemv_phase<MAXB>(c, pi, g);
      tree_phase<MAXB>(c, pi + 1, lp);
    } else {
      g.epi = E_QKV;
      g.o0 = static_cast<__nv_bfloat16*>(p.q);
      g.o1 = static_cast<__nv_bfloat16*>(lp.k_cache);
      g.o2 = static_cast<__nv_bfloat16*>(lp.v_cache);
      gemv_phase<MAXB>(c, pi, g);
      attn_phase(c, lp, sc);
    }
    GemvPhase go{};
    go.epi = E_RESID;
    go.K = d;
    go.N = d;
    go.src = static_cast<const __nv_bfloat16*>(p.y);
    go.x = p.x;
    gemv_phase<MAXB>(c, pi + 2, go);
    GemvPhase gf{};
    gf.epi = E_FFNIN;
    gf.K = d;
    gf.norm_w = static_cast<const __nv_bfloat16*>(lp.norm2);
    gf.o0 = static_cast<__nv_bfloat16*>(p.u);
    gemv_phase<MAXB>(c, pi + 3, gf);
    GemvPhase gd{};
    gd.epi = E_RESID;
    gd.K = p.ff;
    gd.N = d;
    gd.src = static_cast<const __nv_bfloat16*>(p.u);
    gd.x = p.x;
    gemv_phase<MAXB>(c, pi + 4, gd);
  }
  // every position-dependent read of this step is ordered before the next
  // barrier; CTA 0 advances t and the barrier generation once it has passed
  GemvPhase gl{};
  gl.epi = E_LOGITS;
  gl.K = d;
  gl.N = p.vocab;
  gl.norm_w = static_cast<const __nv_bfloat16*>(p.norm_out);
  gl.o0 = static_cast<__nv_bfloat16*>(p.logits);
  gemv_phase<MAXB>(c, 5 * p.n_layers, gl);
  if (c.cta == 0 && threadIdx.x == 0) {
    p.t_buf[0] = c.t + 1;
    atomicAdd(p.barrier + 1, 1ull);
  }
}

template <int MAXB>
int launch_step(const dh_step_params& p, cudaStream_t st) {
  const int kmax = p.ff > p.d ? p.ff : p.d;
  const int xs_elems = ((p.batch * kmax + 7) / 8) * 8;
  const int span = (p.window > 0 && p.window < p.max_len) ? p.window : p.max_len;
  const int chunk = (span + p.nsplit - 1) / p.nsplit;
  const size_t smem = (size_t)kSlots * kSlotBytes + (size_t)xs_elems * 2 + (1280 + (size_t)chunk) * 4;
  DH_REQUIRE(smem <= 227 * 1024, DH_ERR_SHAPE, "dh_decode_step: %zu bytes of shared memory", smem);
  static thread_local int configured_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (configured_dev != dev) {
    cudaFuncSetAttribute(step_kernel<MAXB>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    configured_dev = dev;
  }
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, step_kernel<MAXB>, kThreads, smem);
  DH_REQUIRE(per_sm >= 1, DH_ERR_SHAPE, "dh_decode_step: kernel does not fit on an SM");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sm_count());
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, step_kernel<MAXB>, p, xs_elems) != cudaSuccess)
    return check_launch("step_kernel");
  return DH_OK;
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" int dh_decode_step(const dh_step_params* params, void* stream) {
  DH_REQUIRE(params, DH_ERR_ARG, "dh_decode_step: null params");
  const dh_step_params& p = *params;
  DH_REQUIRE(p.layers && p.tokens && p.t_buf && p.emb && p.norm_out && p.logits && p.x && p.a &&
                 p.v0 && p.y && p.q && p.u && p.ig && p.fg && p.counters && p.barrier && p.status,
             DH_ERR_ARG, "dh_decode_step: null pointer in params");
  DH_REQUIRE(p.batch >= 1 && p.batch <= 16, DH_ERR_SHAPE, "dh_decode_step: batch %d not in [1,16]",
             p.batch);
  DH_REQUIRE(p.hd == 64 && p.d == p.H * p.hd && p.d % 8 == 0 && p.ff % 8 == 0 && p.L >= 1 &&
                 p.L <= 16 && p.nsplit >= 1 && p.n_layers >= 1,
             DH_ERR_SHAPE, "dh_decode_step: unsupported shape (d=%d H=%d hd=%d ff=%d L=%d)", p.d,
             p.H, p.hd, p.ff, p.L);
  DH_REQUIRE(4 * p.ff <= kSlotBytes && 6 * p.d <= kSlotBytes, DH_ERR_SHAPE,
             "dh_decode_step: a weight unit exceeds a stream slot (d=%d ff=%d)", p.d, p.ff);
  DH_REQUIRE(p.nsplit == 1 || p.part, DH_ERR_ARG, "dh_decode_step: nsplit > 1 needs part scratch");
  DH_REQUIRE(p.d <= 1024, DH_ERR_SHAPE, "dh_decode_step: d = %d exceeds 1024", p.d);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (p.batch == 1) return launch_step<1>(p, st);
  if (p.batch == 2) return launch_step<2>(p, st);
  if (p.batch <= 4) return launch_step<4>(p, st);
  if (p.batch <= 8) return launch_step<8>(p, st);
  return launch_step<16>(p, st);
}
