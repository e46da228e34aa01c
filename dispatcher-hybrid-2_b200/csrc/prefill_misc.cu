// Elementwise / row kernels of the parallel forward: embedding gather,
// RMSNorm, RoPE on the q/k projections, and strided row copies that fill the
// decoder caches from the prefill activations.
#include "common.cuh"

namespace dh {
namespace {

constexpr float kEps = 1.1920928955078125e-07f;  // torch RMSNorm eps=None in fp32

// one warp per row; d % 256 == 0 handled with a strided loop of 16-byte chunks
// One warp per row.  CHUNKS > 0: the row is CHUNKS x 256 elements and stays
// in registers (all its loads in flight at once, read once); CHUNKS == 0: any
// D that is a multiple of 8, two passes.  Same summation order either way.
template <int CHUNKS>
__global__ void rmsnorm_kernel(const __nv_bfloat16* x, int ldx, const __nv_bfloat16* w,
                               __nv_bfloat16* y, int ldy, int M, int D) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  const __nv_bfloat16* xr = x + (size_t)warp * ldx;
  float ss = 0.f;
  if constexpr (CHUNKS > 0) {
    uint4 xv[CHUNKS];
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) xv[i] = *reinterpret_cast<const uint4*>(xr + i * 256 + lane * 8);
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      float f[8];
      unpack8(xv[i], f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + kEps);
#pragma unroll
    for (int i = 0; i < CHUNKS; ++i) {
      const int c = i * 256 + lane * 8;
      float f[8], g[8];
      unpack8(xv[i], f);
      unpack8(*reinterpret_cast<const uint4*>(w + c), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = f[e] * r * g[e];
      *reinterpret_cast<uint4*>(y + (size_t)warp * ldy + c) = pack8(f);
    }
  } else {
    for (int c = lane * 8; c < D; c += 256) {
      float f[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + c), f);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss += f[e] * f[e];
    }
    ss = warp_sum(ss);
    const float r = rsqrtf(ss / (float)D + kEps);
    for (int c = lane * 8; c < D; c += 256) {
      float f[8], g[8];
      unpack8(*reinterpret_cast<const uint4*>(xr + c), f);
      unpack8(*reinterpret_cast<const uint4*>(w + c), g);
#pragma unroll
      for (int e = 0; e < 8; ++e) f[e] = f[e] * r * g[e];
      *reinterpret_cast<uint4*>(y + (size_t)warp * ldy + c) = pack8(f);
    }
  }
}

__global__ void embed_rows_kernel(const int64_t* ids, const __nv_bfloat16* emb, __nv_bfloat16* x,
                                  int M, int D, int V, int* status) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= M) return;
  long long tok = ids[warp];
  if (tok < 0 || tok >= V) {
    if (status && lane == 0) atomicExch(status, 1);
    tok = tok < 0 ? 0 : V - 1;
  }
  for (int c = lane * 8; c < D; c += 256)
    *reinterpret_cast<uint4*>(x + (size_t)warp * D + c) =
        *reinterpret_cast<const uint4*>(emb + (size_t)tok * D + c);
}

// rotate pairs (2j, 2j+1) of q and k in place: position of row m is m % T
__global__ void rope_qk_kernel(__nv_bfloat16* p, int ld, int M, int T, int d, int hd,
                               const float* cosT, const float* sinT) {
  const int chunks = (2 * d) / 8;  // q and k, 8 elements per thread
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)M * chunks) return;
  const int m = (int)(idx / chunks), c = (int)(idx % chunks) * 8;
  const int t = m % T;
  __nv_bfloat16* ptr = p + (size_t)m * ld + c;
  float f[8];
  unpack8(*reinterpret_cast<const uint4*>(ptr), f);
  const int j0 = (c % hd) >> 1;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float cs = cosT[(size_t)t * (hd / 2) + j0 + e], sn = sinT[(size_t)t * (hd / 2) + j0 + e];
    const float x1 = f[2 * e], x2 = f[2 * e + 1];
    f[2 * e] = x1 * cs - x2 * sn;
    f[2 * e + 1] = x1 * sn + x2 * cs;
  }
  *reinterpret_cast<uint4*>(ptr) = pack8(f);
}

// dst[b, t, 0:n] = src[b*T + t, 0:n]; dst rows of length ld_dst, batch stride bs_dst
__global__ void copy_rows_kernel(const __nv_bfloat16* src, int ld_src, __nv_bfloat16* dst,
                                 int ld_dst, long long bs_dst, int B, int T, int n) {
  const int chunks = n / 8;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (long long)B * T * chunks) return;
  const long long row = idx / chunks;
  const int c = (int)(idx % chunks) * 8;
  const int b = (int)(row / T), t = (int)(row % T);
  *reinterpret_cast<uint4*>(dst + (size_t)b * bs_dst + (size_t)t * ld_dst + c) =
      *reinterpret_cast<const uint4*>(src + (size_t)row * ld_src + c);
}

}  // namespace
}  // namespace dh

using namespace dh;
#define STREAM(s) reinterpret_cast<cudaStream_t>(s)

extern "C" int dh_rmsnorm_bf16(const void* x, int ldx, const void* w, void* y, int ldy, int M,
                               int D, void* stream) {
  DH_REQUIRE(x && w && y, DH_ERR_ARG, "dh_rmsnorm_bf16: null pointer");
  DH_REQUIRE(D % 8 == 0 && ldx % 8 == 0 && ldy % 8 == 0 && M > 0, DH_ERR_SHAPE,
             "dh_rmsnorm_bf16: bad sizes");
  const int threads = 256, rows_per_block = threads / 32;
  const dim3 grid((M + rows_per_block - 1) / rows_per_block);
  const auto* xp = reinterpret_cast<const __nv_bfloat16*>(x);
  const auto* wp = reinterpret_cast<const __nv_bfloat16*>(w);
  auto* yp = reinterpret_cast<__nv_bfloat16*>(y);
  switch (D % 256 == 0 ? D / 256 : 0) {
    case 1: rmsnorm_kernel<1><<<grid, threads, 0, STREAM(stream)>>>(xp, ldx, wp, yp, ldy, M, D); break;
    case 2: rmsnorm_kernel<2><<<grid, threads, 0, STREAM(stream)>>>(xp, ldx, wp, yp, ldy, M, D); break;
    case 3: rmsnorm_kernel<3><<<grid, threads, 0, STREAM(stream)>>>(xp, ldx, wp, yp, ldy, M, D); break;
    case 4: rmsnorm_kernel<4><<<grid, threads, 0, STREAM(stream)>>>(xp, ldx, wp, yp, ldy, M, D); break;
    default: rmsnorm_kernel<0><<<grid, threads, 0, STREAM(stream)>>>(xp, ldx, wp, yp, ldy, M, D);
  }
  return check_launch("rmsnorm_kernel");
}

extern "C" int dh_embed_bf16(const int64_t* ids, const void* emb, void* x, int M, int D, int V,
                             int* status, void* stream) {
  DH_REQUIRE(ids && emb && x, DH_ERR_ARG, "dh_embed_bf16: null pointer");
  DH_REQUIRE(D % 8 == 0 && M > 0, DH_ERR_SHAPE, "dh_embed_bf16: bad sizes");
  embed_rows_kernel<<<(M + 7) / 8, 256, 0, STREAM(stream)>>>(
      ids, reinterpret_cast<const __nv_bfloat16*>(emb), reinterpret_cast<__nv_bfloat16*>(x), M,
      D, V, status);
  return check_launch("embed_rows_kernel");
}

extern "C" int dh_rope_qk(void* p, int ld, int M, int T, int d, int hd, const float* rope_cos,
                          const float* rope_sin, void* stream) {
  DH_REQUIRE(p && rope_cos && rope_sin, DH_ERR_ARG, "dh_rope_qk: null pointer");
  DH_REQUIRE(hd % 8 == 0 && d % hd == 0 && ld % 8 == 0, DH_ERR_SHAPE, "dh_rope_qk: bad sizes");
  const long long n = (long long)M * (2 * d / 8);
  rope_qk_kernel<<<(unsigned)((n + 255) / 256), 256, 0, STREAM(stream)>>>(
      reinterpret_cast<__nv_bfloat16*>(p), ld, M, T, d, hd, rope_cos, rope_sin);
  return check_launch("rope_qk_kernel");
}

extern "C" int dh_copy_rows(const void* src, int ld_src, void* dst, int ld_dst,
                            long long batch_stride_dst, int batch, int T, int n, void* stream) {
  DH_REQUIRE(src && dst, DH_ERR_ARG, "dh_copy_rows: null pointer");
  DH_REQUIRE(n % 8 == 0 && ld_src % 8 == 0 && ld_dst % 8 == 0 && batch_stride_dst % 8 == 0,
             DH_ERR_SHAPE, "dh_copy_rows: sizes must be multiples of 8 elements");
  const long long total = (long long)batch * T * (n / 8);
  copy_rows_kernel<<<(unsigned)((total + 255) / 256), 256, 0, STREAM(stream)>>>(
      reinterpret_cast<const __nv_bfloat16*>(src), ld_src, reinterpret_cast<__nv_bfloat16*>(dst),
      ld_dst, batch_stride_dst, batch, T, n);
  return check_launch("copy_rows_kernel");
}
