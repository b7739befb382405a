// dcn_simt.cu -- fp32 FFMA (SIMT) deformable-convolution kernels.
//
// These are the strict-parity ("fp32") path of the library and the fallback
// for shapes the tensor-core kernels do not take.  Every GEMM is an implicit
// GEMM: the deformable column buffer of the reference
// (deform_conv2d.metal:74-125) is never materialised; its tiles are gathered
// straight into shared memory from the NHWC copy of the input.
//
//   forward   out[n, o, p]  = bias[o] + sum_{k,c} W[o, c, k] col[n, c, k, p]
//   grad col  gcol[n,c,k,p] = sum_o W[o, c, k] go[n, o, p]      (.mm:820-821)
//             -> fused col2im scatter       (deform_conv2d.metal:141-204)
//             -> fused coordinate reduction (deform_conv2d.metal:225-295)
//   grad W    gW[o, c, k]   = sum_{n,p} go[n, o, p] col[n, c, k, p] (.mm:880)
//
// K is ordered (tap k, channel c) so that the bilinear sampling plan of one
// (pixel, tap) is computed once and reused for every channel of the tap.
#include "dcn_kernels.h"

namespace dcn {

namespace {

// Loads the sampling plan of (image n, pixel p = (oy, ox), tap k, deformable
// group dgi) and the modulation scalar.
__device__ __forceinline__ Sample load_sample(const Geom& g, const float* __restrict__ off,
                                              const float* __restrict__ mask, int n, int p,
                                              int oy, int ox, int k, int dgi, float& m) {
  const int ki = k / g.kw, kj = k - ki * g.kw;
  const long long oi = off_h_index(g, n, dgi, k, p);
  const float offh = __ldg(off + oi), offw = __ldg(off + oi + g.P);
  float h, w;
  sample_pos(g, oy, ox, ki, kj, offh, offw, h, w);
  m = mask_of(g, mask, mask_index(g, n, dgi, k, p));
  return make_sample(h, w, g.H, g.W);
}

__device__ __forceinline__ float4 ld4_live(const float* p, bool live) {
  return live ? ldg4(p) : make_float4(0.f, 0.f, 0.f, 0.f);
}
__device__ __forceinline__ float ld1_live(const float* p, bool live) {
  return live ? __ldg(p) : 0.f;
}

__device__ __forceinline__ float f4get(const float4& v, int j) {
  return j == 0 ? v.x : (j == 1 ? v.y : (j == 2 ? v.z : v.w));
}

// ===========================================================================
// Forward implicit GEMM.  CTA tile: 128 output pixels (flattened n*P + p) x
// 128 output channels of one group; K step: 8 channels of one tap.
// 256 threads, 8x8 accumulators each; register-staged double buffering.
// VEC: C, Cg and C/dg are multiples of 4, so a thread's 4 channels share one
// sampling plan and are read with one 16-byte load per corner.
// ===========================================================================
constexpr int F_BM = 128, F_BN = 128, F_BK = 8, F_PAD = 4;

template <bool VEC>
__global__ void __launch_bounds__(256, 2)
fwd_simt_gemm_kernel(Geom g, const float* __restrict__ xt, const float* __restrict__ wf,
                     int cpad, const float* __restrict__ off, const float* __restrict__ mask,
                     const float* __restrict__ bias, float* __restrict__ out) {
  __shared__ __align__(16) float As[2][F_BK][F_BM + F_PAD];
  __shared__ __align__(16) float Bs[2][F_BK][F_BN + F_PAD];

  const int tid = threadIdx.x;
  const long long q0 = (long long)blockIdx.x * F_BM;
  const int o0 = blockIdx.y * F_BN;
  const int gi = blockIdx.z;
  const int nchunk = cpad / F_BK;
  const int steps = g.kk * nchunk;

  // ---- gather role: pixel gm, channels ghalf*4 .. +3 of each K step ----
  const int gm = tid >> 1, ghalf = tid & 1;
  const long long gq = q0 + gm;
  const bool gq_ok = gq < g.NP;
  int gn = 0, gp = 0, goy = 0, gox = 0;
  if (gq_ok) {
    gn = (int)(gq / g.P);
    gp = (int)(gq - (long long)gn * g.P);
    goy = gp / g.Wo;
    gox = gp - goy * g.Wo;
  }
  const float* xt_n = xt + (long long)gn * g.HW * g.C;

  int cached_k = -1, cached_dgi = -1;
  Sample smp = make_sample(-2.f, -2.f, 1, 1);
  float smask = 0.f;
  // raw corner values of the next step (VEC: 4 corners x float4)
  float4 r1, r2, r3, r4;
  float sv[4];  // scalar path: finished values
  float breg[4];

  auto load = [&](int step) {
    const int k = step / nchunk;
    const int c0 = (step - k * nchunk) * F_BK;
    const int cb = c0 + ghalf * 4;
    if constexpr (VEC) {
      r1 = r2 = r3 = r4 = make_float4(0.f, 0.f, 0.f, 0.f);
      if (gq_ok && cb < g.Cg) {
        const int gch = gi * g.Cg + cb;
        const int dgi = gch / g.cpg;
        if (k != cached_k || dgi != cached_dgi) {
          smp = load_sample(g, off, mask, gn, gp, goy, gox, k, dgi, smask);
          cached_k = k;
          cached_dgi = dgi;
        }
        if (smp.valid) {
          const float* base = xt_n + gch;
          r1 = ld4_live(base + (long long)smp.i1 * g.C, smp.live & 1u);
          r2 = ld4_live(base + (long long)smp.i2 * g.C, smp.live & 2u);
          r3 = ld4_live(base + (long long)smp.i3 * g.C, smp.live & 4u);
          r4 = ld4_live(base + (long long)smp.i4 * g.C, smp.live & 8u);
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        sv[j] = 0.f;
        const int c = cb + j;
        if (gq_ok && c < g.Cg) {
          const int gch = gi * g.Cg + c;
          const int dgi = gch / g.cpg;
          if (k != cached_k || dgi != cached_dgi) {
            smp = load_sample(g, off, mask, gn, gp, goy, gox, k, dgi, smask);
            cached_k = k;
            cached_dgi = dgi;
          }
          if (smp.valid) {
            const float* base = xt_n + gch;
            const float v1 = ld1_live(base + (long long)smp.i1 * g.C, smp.live & 1u);
            const float v2 = ld1_live(base + (long long)smp.i2 * g.C, smp.live & 2u);
            const float v3 = ld1_live(base + (long long)smp.i3 * g.C, smp.live & 4u);
            const float v4 = ld1_live(base + (long long)smp.i4 * g.C, smp.live & 8u);
            sv[j] = bilerp(smp, v1, v2, v3, v4) * smask;
          }
        }
      }
    }
    const float* wrow = wf + ((long long)(gi * g.kk + k) * cpad + c0) * g.Og;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int idx = tid + 256 * j;
      const int row = idx >> 7, col = idx & 127;
      const int o = o0 + col;
      breg[j] = (o < g.Og) ? __ldg(wrow + (long long)row * g.Og + o) : 0.f;
    }
  };

  auto store = [&](int buf) {
    if constexpr (VEC) {
      const float m = smp.valid ? smask : 0.f;
      As[buf][ghalf * 4 + 0][gm] = bilerp(smp, r1.x, r2.x, r3.x, r4.x) * m;
      As[buf][ghalf * 4 + 1][gm] = bilerp(smp, r1.y, r2.y, r3.y, r4.y) * m;
      As[buf][ghalf * 4 + 2][gm] = bilerp(smp, r1.z, r2.z, r3.z, r4.z) * m;
      As[buf][ghalf * 4 + 3][gm] = bilerp(smp, r1.w, r2.w, r3.w, r4.w) * m;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j) As[buf][ghalf * 4 + j][gm] = sv[j];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int idx = tid + 256 * j;
      Bs[buf][idx >> 7][idx & 127] = breg[j];
    }
  };

  const int tm = tid & 15, tn = tid >> 4;
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  load(0);
  store(0);
  __syncthreads();
  for (int s = 0; s < steps; ++s) {
    const int cur = s & 1;
    if (s + 1 < steps) load(s + 1);
#pragma unroll
    for (int kk = 0; kk < F_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][tm * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + tm * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tn * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tn * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (s + 1 < steps) store(cur ^ 1);
    __syncthreads();
  }

  // ---- epilogue: bias, NCHW store ----
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = (i < 4) ? tm * 4 + i : 64 + tm * 4 + (i - 4);
    const long long q = q0 + m;
    if (q >= g.NP) continue;
    const int n = (int)(q / g.P);
    const int p = (int)(q - (long long)n * g.P);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int ol = (j < 4) ? tn * 4 + j : 64 + tn * 4 + (j - 4);
      const int o = o0 + ol;
      if (o >= g.Og) continue;
      const int oc = gi * g.Og + o;
      const float b = (g.use_bias) ? __ldg(bias + oc) : 0.f;
      out[((long long)n * g.outC + oc) * g.P + p] = acc[i][j] + b;
    }
  }
}

// ===========================================================================
// Forward, direct form for small groups (out channels per group <= 8): one
// thread per (pixel, group), all of the group's weights in shared memory.
// ===========================================================================
constexpr int D_THREADS = 128;
constexpr int DIRECT_MAX_OG = 8;
constexpr int DIRECT_MAX_SMEM = 48 * 1024;

template <int OG>
__global__ void __launch_bounds__(D_THREADS)
fwd_simt_direct_kernel(Geom g, const float* __restrict__ xt, const float* __restrict__ w,
                       const float* __restrict__ off, const float* __restrict__ mask,
                       const float* __restrict__ bias, float* __restrict__ out) {
  extern __shared__ float ws[];  // [Og][Cg][kk] of group gi
  const int gi = blockIdx.y;
  const int wcount = g.Og * g.Cg * g.kk;
  for (int i = threadIdx.x; i < wcount; i += D_THREADS)
    ws[i] = w[(long long)gi * wcount + i];
  __syncthreads();

  const long long q = (long long)blockIdx.x * D_THREADS + threadIdx.x;
  if (q >= g.NP) return;
  const int n = (int)(q / g.P);
  const int p = (int)(q - (long long)n * g.P);
  const int oy = p / g.Wo, ox = p - oy * g.Wo;
  const float* xt_n = xt + (long long)n * g.HW * g.C;

  float acc[OG];
#pragma unroll
  for (int o = 0; o < OG; ++o) acc[o] = 0.f;

  for (int k = 0; k < g.kk; ++k) {
    int cached_dgi = -1;
    Sample smp = make_sample(-2.f, -2.f, 1, 1);
    float m = 0.f;
    for (int c = 0; c < g.Cg; ++c) {
      const int gch = gi * g.Cg + c;
      const int dgi = gch / g.cpg;
      if (dgi != cached_dgi) {
        smp = load_sample(g, off, mask, n, p, oy, ox, k, dgi, m);
        cached_dgi = dgi;
      }
      if (!smp.valid) continue;
      const float* base = xt_n + gch;
      const float v1 = ld1_live(base + (long long)smp.i1 * g.C, smp.live & 1u);
      const float v2 = ld1_live(base + (long long)smp.i2 * g.C, smp.live & 2u);
      const float v3 = ld1_live(base + (long long)smp.i3 * g.C, smp.live & 4u);
      const float v4 = ld1_live(base + (long long)smp.i4 * g.C, smp.live & 8u);
      const float val = bilerp(smp, v1, v2, v3, v4) * m;
#pragma unroll
      for (int o = 0; o < OG; ++o)
        if (o < g.Og) acc[o] = fmaf(ws[(o * g.Cg + c) * g.kk + k], val, acc[o]);
    }
  }
#pragma unroll
  for (int o = 0; o < OG; ++o) {
    if (o >= g.Og) break;
    const int oc = gi * g.Og + o;
    const float b = g.use_bias ? __ldg(bias + oc) : 0.f;
    out[((long long)n * g.outC + oc) * g.P + p] = acc[o] + b;
  }
}

// ===========================================================================
// Backward data path.  CTA: 128 pixels x 64 channels of one group at one tap;
// K = out channels of the group (8 per step).  The grad-column tile lives in
// registers (8 pixels x 4 channels per thread) and is consumed in place:
//  * col2im: scatter gcol * mask * corner weight into the NHWC grad-input
//    accumulator with 16-byte vector reductions;
//  * coordinate / mask gradients: per-thread partial sums over its channels,
//    reduced across the 16 lanes that share a pixel with warp shuffles, one
//    atomic per (pixel, tap) per CTA.
// ===========================================================================
constexpr int B_BM = 128, B_BN = 64, B_BK = 8;

template <bool VEC>
__global__ void __launch_bounds__(256, 2)
bwd_data_simt_kernel(Geom g, const float* __restrict__ go, const float* __restrict__ wb,
                     const float* __restrict__ xt, const float* __restrict__ off,
                     const float* __restrict__ mask, float* __restrict__ gxt,
                     float* __restrict__ goff, float* __restrict__ gmask) {
  __shared__ __align__(16) float As[2][B_BK][B_BM + 4];  // go  [o][pixel]
  __shared__ __align__(16) float Bs[2][B_BK][B_BN + 4];  // W   [o][channel]

  const int tid = threadIdx.x;
  const long long q0 = (long long)blockIdx.x * B_BM;
  const int nct = ceil_div(g.Cg, B_BN);
  const int k = blockIdx.y / nct;
  const int c0 = (blockIdx.y - k * nct) * B_BN;
  const int gi = blockIdx.z;
  const int steps = ceil_div(g.Og, B_BK);

  // A loader: row = tid / 32 (out channel within step), 4 pixels per thread
  const int arow = tid >> 5;
  const float* abase[4];
  bool aok[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const long long q = q0 + (tid & 31) + 32 * j;
    aok[j] = q < g.NP;
    int n = 0, p = 0;
    if (aok[j]) {
      n = (int)(q / g.P);
      p = (int)(q - (long long)n * g.P);
    }
    abase[j] = go + ((long long)n * g.outC + (long long)gi * g.Og) * g.P + p;
  }
  const float* wrow = wb + (long long)(gi * g.kk + k) * g.Og * g.Cg;

  float areg[4], breg[2];
  auto load = [&](int s) {
    const int o = s * B_BK + arow;
#pragma unroll
    for (int j = 0; j < 4; ++j) areg[j] = (aok[j] && o < g.Og) ? __ldg(abase[j] + (long long)o * g.P) : 0.f;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int c = c0 + (tid & 31) + 32 * j;
      breg[j] = (o < g.Og && c < g.Cg) ? __ldg(wrow + (long long)o * g.Cg + c) : 0.f;
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 4; ++j) As[buf][arow][(tid & 31) + 32 * j] = areg[j];
#pragma unroll
    for (int j = 0; j < 2; ++j) Bs[buf][arow][(tid & 31) + 32 * j] = breg[j];
  };

  const int tm = tid >> 4, tn = tid & 15;
  float acc[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  load(0);
  store(0);
  __syncthreads();
  for (int s = 0; s < steps; ++s) {
    const int cur = s & 1;
    if (s + 1 < steps) load(s + 1);
#pragma unroll
    for (int kk = 0; kk < B_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][tm * 4]);
      const float4 a1 = *reinterpret_cast<const float4*>(&As[cur][kk][64 + tm * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tn * 4]);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float b[4] = {b0.x, b0.y, b0.z, b0.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (s + 1 < steps) store(cur ^ 1);
    __syncthreads();
  }

  // ---- epilogue: col2im scatter + coordinate / mask reductions ----
  const int cfirst = gi * g.Cg + c0;
  const int clast = gi * g.Cg + min(c0 + B_BN, g.Cg) - 1;
  const bool uniform_dg = (cfirst / g.cpg) == (clast / g.cpg);
  const int cb = c0 + tn * 4;

#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int m = (i < 4) ? tm * 4 + i : 64 + tm * 4 + (i - 4);
    const long long q = q0 + m;
    const bool ok = q < g.NP;
    int n = 0, p = 0, oy = 0, ox = 0;
    if (ok) {
      n = (int)(q / g.P);
      p = (int)(q - (long long)n * g.P);
      oy = p / g.Wo;
      ox = p - oy * g.Wo;
    }
    const float* xt_n = xt + (long long)n * g.HW * g.C;
    float* gxt_n = gxt + (long long)n * g.HW * g.C;
    float s_h = 0.f, s_w = 0.f, s_m = 0.f;
    if constexpr (VEC) {
      if (ok && cb < g.Cg) {
        const int gch = gi * g.Cg + cb;
        const int dgi = gch / g.cpg;
        float msk;
        const Sample smp = load_sample(g, off, mask, n, p, oy, ox, k, dgi, msk);
        if (smp.valid) {
          const float* base = xt_n + gch;
          const float4 v1 = ld4_live(base + (long long)smp.i1 * g.C, smp.live & 1u);
          const float4 v2 = ld4_live(base + (long long)smp.i2 * g.C, smp.live & 2u);
          const float4 v3 = ld4_live(base + (long long)smp.i3 * g.C, smp.live & 4u);
          const float4 v4 = ld4_live(base + (long long)smp.i4 * g.C, smp.live & 8u);
          float top[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float a = f4get(v1, j), b = f4get(v2, j), c = f4get(v3, j), d = f4get(v4, j);
            const float gc = acc[i][j];
            s_h += msk * coord_dh(smp, a, b, c, d) * gc;
            s_w += msk * coord_dw(smp, a, b, c, d) * gc;
            s_m += gc * bilerp(smp, a, b, c, d);
            top[j] = gc * msk;
          }
          s_m *= mask_grad_scale(g, msk);  // per pixel: scales every lane's partial alike
          float* gbase = gxt_n + gch;
          if (smp.live & 1u)
            red_add_v4(gbase + (long long)smp.i1 * g.C, smp.w1 * top[0], smp.w1 * top[1],
                       smp.w1 * top[2], smp.w1 * top[3]);
          if (smp.live & 2u)
            red_add_v4(gbase + (long long)smp.i2 * g.C, smp.w2 * top[0], smp.w2 * top[1],
                       smp.w2 * top[2], smp.w2 * top[3]);
          if (smp.live & 4u)
            red_add_v4(gbase + (long long)smp.i3 * g.C, smp.w3 * top[0], smp.w3 * top[1],
                       smp.w3 * top[2], smp.w3 * top[3]);
          if (smp.live & 8u)
            red_add_v4(gbase + (long long)smp.i4 * g.C, smp.w4 * top[0], smp.w4 * top[1],
                       smp.w4 * top[2], smp.w4 * top[3]);
          if (!uniform_dg) {
            const long long oi = off_h_index(g, n, dgi, k, p);
            red_add_f32(goff + oi, s_h);
            red_add_f32(goff + oi + g.P, s_w);
            if (g.use_mask) red_add_f32(gmask + mask_index(g, n, dgi, k, p), s_m);
          }
        }
      }
      if (uniform_dg) {
#pragma unroll
        for (int d = 8; d > 0; d >>= 1) {
          s_h += __shfl_xor_sync(0xffffffffu, s_h, d);
          s_w += __shfl_xor_sync(0xffffffffu, s_w, d);
          s_m += __shfl_xor_sync(0xffffffffu, s_m, d);
        }
        if (tn == 0 && ok) {
          const int dgi = cfirst / g.cpg;
          const long long oi = off_h_index(g, n, dgi, k, p);
          red_add_f32(goff + oi, s_h);
          red_add_f32(goff + oi + g.P, s_w);
          if (g.use_mask) red_add_f32(gmask + mask_index(g, n, dgi, k, p), s_m);
        }
      }
    } else {
      // general shapes: one sampling plan per channel, per-channel atomics
      if (ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int c = cb + j;
          if (c >= g.Cg) break;
          const int gch = gi * g.Cg + c;
          const int dgi = gch / g.cpg;
          float msk;
          const Sample smp = load_sample(g, off, mask, n, p, oy, ox, k, dgi, msk);
          if (!smp.valid) continue;
          const float* base = xt_n + gch;
          const float a = ld1_live(base + (long long)smp.i1 * g.C, smp.live & 1u);
          const float b = ld1_live(base + (long long)smp.i2 * g.C, smp.live & 2u);
          const float cc = ld1_live(base + (long long)smp.i3 * g.C, smp.live & 4u);
          const float d = ld1_live(base + (long long)smp.i4 * g.C, smp.live & 8u);
          const float gc = acc[i][j];
          const long long oi = off_h_index(g, n, dgi, k, p);
          red_add_f32(goff + oi, msk * coord_dh(smp, a, b, cc, d) * gc);
          red_add_f32(goff + oi + g.P, msk * coord_dw(smp, a, b, cc, d) * gc);
          if (g.use_mask)
            red_add_f32(gmask + mask_index(g, n, dgi, k, p),
                        gc * bilerp(smp, a, b, cc, d) * mask_grad_scale(g, msk));
          const float top = gc * msk;
          float* gbase = gxt_n + gch;
          if (smp.live & 1u) red_add_f32(gbase + (long long)smp.i1 * g.C, smp.w1 * top);
          if (smp.live & 2u) red_add_f32(gbase + (long long)smp.i2 * g.C, smp.w2 * top);
          if (smp.live & 4u) red_add_f32(gbase + (long long)smp.i3 * g.C, smp.w3 * top);
          if (smp.live & 8u) red_add_f32(gbase + (long long)smp.i4 * g.C, smp.w4 * top);
        }
      }
    }
  }
}

// ===========================================================================
// grad_weight: M = out channels of a group (64 per CTA), N = 128 channels of
// one tap, K = pixels (16 per step), split-K over the pixel range; partial
// tiles are reduced with fp32 atomics into the pre-zeroed grad_weight.
// VEC: Cg and C/dg are multiples of 8 and C of 4.
// ===========================================================================
constexpr int W_BM = 64, W_BN = 128, W_BK = 16;

template <bool VEC>
__global__ void __launch_bounds__(256, 2)
bwd_weight_simt_kernel(Geom g, const float* __restrict__ go, const float* __restrict__ xt,
                       const float* __restrict__ off, const float* __restrict__ mask,
                       float* __restrict__ gw, int splits, long long q_per_split) {
  __shared__ __align__(16) float As[2][W_BK][W_BM + 4];  // go  [pixel][o]
  __shared__ __align__(16) float Bs[2][W_BK][W_BN + 4];  // col [pixel][c]

  const int tid = threadIdx.x;
  const int o0 = blockIdx.x * W_BM;
  const int nct = ceil_div(g.Cg, W_BN);
  const int k = blockIdx.y / nct;
  const int c0 = (blockIdx.y - k * nct) * W_BN;
  const int gi = blockIdx.z / splits;
  const int split = blockIdx.z - gi * splits;
  const long long qb = (long long)split * q_per_split;
  const long long qe = min(g.NP, qb + q_per_split);
  if (qb >= qe) return;
  const int steps = (int)((qe - qb + W_BK - 1) / W_BK);

  // A loader: pixel apx = tid & 15, out channels (tid >> 4) + 16 j
  const int apx = tid & 15, aoc = tid >> 4;
  // B loader: pixel bpx = tid >> 4, channels bcb .. bcb + 7
  const int bpx = tid >> 4, bcb = (tid & 15) * 8;

  float areg[4];
  float bval[8];
  auto load = [&](int s) {
    {
      const long long q = qb + (long long)s * W_BK + apx;
      const bool ok = q < qe;
      int n = 0, p = 0;
      if (ok) {
        n = (int)(q / g.P);
        p = (int)(q - (long long)n * g.P);
      }
      const float* base = go + ((long long)n * g.outC + (long long)gi * g.Og) * g.P + p;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int o = o0 + aoc + 16 * j;
        areg[j] = (ok && o < g.Og) ? __ldg(base + (long long)o * g.P) : 0.f;
      }
    }
    {
      const long long q = qb + (long long)s * W_BK + bpx;
#pragma unroll
      for (int j = 0; j < 8; ++j) bval[j] = 0.f;
      if (q < qe) {
        const int n = (int)(q / g.P);
        const int p = (int)(q - (long long)n * g.P);
        const int oy = p / g.Wo, ox = p - oy * g.Wo;
        const float* xt_n = xt + (long long)n * g.HW * g.C;
        if constexpr (VEC) {
          const int cb = c0 + bcb;
          if (cb < g.Cg) {
            const int gch = gi * g.Cg + cb;
            float msk;
            const Sample smp = load_sample(g, off, mask, n, p, oy, ox, k, gch / g.cpg, msk);
            if (smp.valid) {
              const float* base = xt_n + gch;
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                const float4 v1 = ld4_live(base + (long long)smp.i1 * g.C + 4 * h, smp.live & 1u);
                const float4 v2 = ld4_live(base + (long long)smp.i2 * g.C + 4 * h, smp.live & 2u);
                const float4 v3 = ld4_live(base + (long long)smp.i3 * g.C + 4 * h, smp.live & 4u);
                const float4 v4 = ld4_live(base + (long long)smp.i4 * g.C + 4 * h, smp.live & 8u);
                bval[4 * h + 0] = bilerp(smp, v1.x, v2.x, v3.x, v4.x) * msk;
                bval[4 * h + 1] = bilerp(smp, v1.y, v2.y, v3.y, v4.y) * msk;
                bval[4 * h + 2] = bilerp(smp, v1.z, v2.z, v3.z, v4.z) * msk;
                bval[4 * h + 3] = bilerp(smp, v1.w, v2.w, v3.w, v4.w) * msk;
              }
            }
          }
        } else {
          int cached_dgi = -1;
          Sample smp = make_sample(-2.f, -2.f, 1, 1);
          float msk = 0.f;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int c = c0 + bcb + j;
            if (c >= g.Cg) break;
            const int gch = gi * g.Cg + c;
            const int dgi = gch / g.cpg;
            if (dgi != cached_dgi) {
              smp = load_sample(g, off, mask, n, p, oy, ox, k, dgi, msk);
              cached_dgi = dgi;
            }
            if (!smp.valid) continue;
            const float* base = xt_n + gch;
            const float v1 = ld1_live(base + (long long)smp.i1 * g.C, smp.live & 1u);
            const float v2 = ld1_live(base + (long long)smp.i2 * g.C, smp.live & 2u);
            const float v3 = ld1_live(base + (long long)smp.i3 * g.C, smp.live & 4u);
            const float v4 = ld1_live(base + (long long)smp.i4 * g.C, smp.live & 8u);
            bval[j] = bilerp(smp, v1, v2, v3, v4) * msk;
          }
        }
      }
    }
  };
  auto store = [&](int buf) {
#pragma unroll
    for (int j = 0; j < 4; ++j) As[buf][apx][aoc + 16 * j] = areg[j];
    *reinterpret_cast<float4*>(&Bs[buf][bpx][bcb]) = make_float4(bval[0], bval[1], bval[2], bval[3]);
    *reinterpret_cast<float4*>(&Bs[buf][bpx][bcb + 4]) = make_float4(bval[4], bval[5], bval[6], bval[7]);
  };

  const int tm = tid >> 4, tn = tid & 15;
  float acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

  load(0);
  store(0);
  __syncthreads();
  for (int s = 0; s < steps; ++s) {
    const int cur = s & 1;
    if (s + 1 < steps) load(s + 1);
#pragma unroll
    for (int kk = 0; kk < W_BK; ++kk) {
      const float4 a0 = *reinterpret_cast<const float4*>(&As[cur][kk][tm * 4]);
      const float4 b0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tn * 4]);
      const float4 b1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][64 + tn * 4]);
      const float a[4] = {a0.x, a0.y, a0.z, a0.w};
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
    }
    if (s + 1 < steps) store(cur ^ 1);
    __syncthreads();
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int o = o0 + tm * 4 + i;
    if (o >= g.Og) continue;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = c0 + ((j < 4) ? tn * 4 + j : 64 + tn * 4 + (j - 4));
      if (c >= g.Cg) continue;
      red_add_f32(gw + ((long long)(gi * g.Og + o) * g.Cg + c) * g.kk + k, acc[i][j]);
    }
  }
}

// ===========================================================================
// Backward for small groups (<= 8 out channels and <= 16 in channels per
// group, e.g. groups=32 with 2 channels each).  One thread per (pixel, group)
// does the whole backward of its pixel for that group: the grad-column values
// (a tiny K = Og dot product), the col2im scatter, the coordinate / mask sums
// of its channels (atomics, since other groups share the deformable group),
// and its contribution to grad_weight, first summed over the block's pixels
// in shared memory.  Block = 128 pixels of one group.
// ===========================================================================
constexpr int SMALL_THREADS = 128;
constexpr int SMALL_MAX_OG = 8, SMALL_MAX_CG = 16;

template <int OG>
__global__ void __launch_bounds__(SMALL_THREADS)
bwd_small_kernel(Geom g, const float* __restrict__ go, const float* __restrict__ w,
                 const float* __restrict__ xt, const float* __restrict__ off,
                 const float* __restrict__ mask, float* __restrict__ gxt,
                 float* __restrict__ goff, float* __restrict__ gmask, float* __restrict__ gw) {
  extern __shared__ float sm[];  // [Og][Cg][kk] weights, then the same size of grad_weight sums
  const int gi = blockIdx.y;
  const int wcount = g.Og * g.Cg * g.kk;
  float* ws = sm;
  float* gws = sm + wcount;
  for (int i = threadIdx.x; i < wcount; i += SMALL_THREADS) {
    ws[i] = w[(long long)gi * wcount + i];
    gws[i] = 0.f;
  }
  __syncthreads();
  const long long q = (long long)blockIdx.x * SMALL_THREADS + threadIdx.x;
  if (q < g.NP) {
    const int n = (int)(q / g.P);
    const int p = (int)(q - (long long)n * g.P);
    const int oy = p / g.Wo, ox = p - oy * g.Wo;
    float gov[OG];
#pragma unroll
    for (int o = 0; o < OG; ++o)
      gov[o] = o < g.Og ? __ldg(go + ((long long)n * g.outC + gi * g.Og + o) * g.P + p) : 0.f;
    const float* xt_n = xt + (long long)n * g.HW * g.C;
    float* gxt_n = gxt + (long long)n * g.HW * g.C;
    for (int k = 0; k < g.kk; ++k) {
      const int ki = k / g.kw, kj = k - ki * g.kw;
      int cur_dgi = -1;
      Sample sp = make_sample(-2.f, -2.f, 1, 1);
      float msk = 0.f, s_h = 0.f, s_w = 0.f, s_m = 0.f;
      for (int c = 0; c < g.Cg; ++c) {
        const int gch = gi * g.Cg + c;
        const int dgi = gch / g.cpg;
        if (dgi != cur_dgi) {
          if (cur_dgi >= 0 && sp.valid) {
            const long long oi = off_h_index(g, n, cur_dgi, k, p);
            red_add_f32(goff + oi, s_h);
            red_add_f32(goff + oi + g.P, s_w);
            if (g.use_mask)
              red_add_f32(gmask + mask_index(g, n, cur_dgi, k, p), s_m * mask_grad_scale(g, msk));
          }
          s_h = s_w = s_m = 0.f;
          cur_dgi = dgi;
          const long long oi = off_h_index(g, n, dgi, k, p);
          float h, wv;
          sample_pos(g, oy, ox, ki, kj, __ldg(off + oi), __ldg(off + oi + g.P), h, wv);
          msk = mask_of(g, mask, mask_index(g, n, dgi, k, p));
          sp = make_sample(h, wv, g.H, g.W);
        }
        if (!sp.valid) continue;
        float gc = 0.f;
#pragma unroll
        for (int o = 0; o < OG; ++o)
          if (o < g.Og) gc = fmaf(gov[o], ws[(o * g.Cg + c) * g.kk + k], gc);
        const float* base = xt_n + gch;
        const float a = (sp.live & 1u) ? __ldg(base + (long long)sp.i1 * g.C) : 0.f;
        const float b = (sp.live & 2u) ? __ldg(base + (long long)sp.i2 * g.C) : 0.f;
        const float cc = (sp.live & 4u) ? __ldg(base + (long long)sp.i3 * g.C) : 0.f;
        const float d = (sp.live & 8u) ? __ldg(base + (long long)sp.i4 * g.C) : 0.f;
        const float val = bilerp(sp, a, b, cc, d);
        s_h += msk * coord_dh(sp, a, b, cc, d) * gc;
        s_w += msk * coord_dw(sp, a, b, cc, d) * gc;
        s_m += gc * val;
        const float top = gc * msk;
        float* gb = gxt_n + gch;
        if (sp.live & 1u) red_add_f32(gb + (long long)sp.i1 * g.C, sp.w1 * top);
        if (sp.live & 2u) red_add_f32(gb + (long long)sp.i2 * g.C, sp.w2 * top);
        if (sp.live & 4u) red_add_f32(gb + (long long)sp.i3 * g.C, sp.w3 * top);
        if (sp.live & 8u) red_add_f32(gb + (long long)sp.i4 * g.C, sp.w4 * top);
        const float colv = val * msk;
#pragma unroll
        for (int o = 0; o < OG; ++o)
          if (o < g.Og) atomicAdd(&gws[(o * g.Cg + c) * g.kk + k], gov[o] * colv);
      }
      if (cur_dgi >= 0 && sp.valid) {
        const long long oi = off_h_index(g, n, cur_dgi, k, p);
        red_add_f32(goff + oi, s_h);
        red_add_f32(goff + oi + g.P, s_w);
        if (g.use_mask)
          red_add_f32(gmask + mask_index(g, n, cur_dgi, k, p), s_m * mask_grad_scale(g, msk));
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < wcount; i += SMALL_THREADS)
    red_add_f32(gw + (long long)gi * wcount + i, gws[i]);
}

bool vec4_ok(const Geom& g) { return g.C % 4 == 0 && g.Cg % 4 == 0 && g.cpg % 4 == 0; }
bool vec8_ok(const Geom& g) { return g.C % 4 == 0 && g.Cg % 8 == 0 && g.cpg % 8 == 0; }

}  // namespace

cudaError_t launch_fwd_simt_gemm(const Geom& g, const float* xt, const float* wf, int cpad,
                                 const float* off, const float* mask, const float* bias,
                                 float* out, cudaStream_t stream) {
  if (g.NP == 0 || g.outC == 0) return cudaSuccess;
  dim3 grid((unsigned)((g.NP + F_BM - 1) / F_BM), ceil_div(g.Og, F_BN), g.G);
  if (vec4_ok(g))
    fwd_simt_gemm_kernel<true><<<grid, 256, 0, stream>>>(g, xt, wf, cpad, off, mask, bias, out);
  else
    fwd_simt_gemm_kernel<false><<<grid, 256, 0, stream>>>(g, xt, wf, cpad, off, mask, bias, out);
  return cudaGetLastError();
}

bool fwd_direct_supported(const Geom& g) {
  return g.Og <= DIRECT_MAX_OG &&
         (long long)g.Og * g.Cg * g.kk * sizeof(float) <= DIRECT_MAX_SMEM;
}

cudaError_t launch_fwd_simt_direct(const Geom& g, const float* xt, const float* w,
                                   const float* off, const float* mask, const float* bias,
                                   float* out, cudaStream_t stream) {
  if (g.NP == 0 || g.outC == 0) return cudaSuccess;
  if (!fwd_direct_supported(g)) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((g.NP + D_THREADS - 1) / D_THREADS), g.G);
  const size_t smem = (size_t)g.Og * g.Cg * g.kk * sizeof(float);
  if (g.Og <= 1)
    fwd_simt_direct_kernel<1><<<grid, D_THREADS, smem, stream>>>(g, xt, w, off, mask, bias, out);
  else if (g.Og <= 2)
    fwd_simt_direct_kernel<2><<<grid, D_THREADS, smem, stream>>>(g, xt, w, off, mask, bias, out);
  else if (g.Og <= 4)
    fwd_simt_direct_kernel<4><<<grid, D_THREADS, smem, stream>>>(g, xt, w, off, mask, bias, out);
  else
    fwd_simt_direct_kernel<8><<<grid, D_THREADS, smem, stream>>>(g, xt, w, off, mask, bias, out);
  return cudaGetLastError();
}

cudaError_t launch_bwd_data_simt(const Geom& g, const float* go, const float* wb,
                                 const float* xt, const float* off, const float* mask,
                                 float* gxt, float* goff, float* gmask, cudaStream_t stream) {
  if (g.NP == 0 || g.Cg == 0 || g.Og == 0) return cudaSuccess;
  dim3 grid((unsigned)((g.NP + B_BM - 1) / B_BM), g.kk * ceil_div(g.Cg, B_BN), g.G);
  if (vec4_ok(g))
    bwd_data_simt_kernel<true><<<grid, 256, 0, stream>>>(g, go, wb, xt, off, mask, gxt, goff, gmask);
  else
    bwd_data_simt_kernel<false><<<grid, 256, 0, stream>>>(g, go, wb, xt, off, mask, gxt, goff, gmask);
  return cudaGetLastError();
}

bool bwd_small_supported(const Geom& g) {
  return g.Og <= SMALL_MAX_OG && g.Cg <= SMALL_MAX_CG &&
         (size_t)2 * g.Og * g.Cg * g.kk * sizeof(float) <= 48 * 1024;
}

cudaError_t launch_bwd_small(const Geom& g, const float* go, const float* w, const float* xt,
                             const float* off, const float* mask, float* gxt, float* goff,
                             float* gmask, float* gw, cudaStream_t stream) {
  if (g.NP == 0 || g.Cg == 0 || g.Og == 0) return cudaSuccess;
  if (!bwd_small_supported(g)) return cudaErrorInvalidValue;
  dim3 grid((unsigned)((g.NP + SMALL_THREADS - 1) / SMALL_THREADS), g.G);
  const size_t smem = (size_t)2 * g.Og * g.Cg * g.kk * sizeof(float);
  if (g.Og <= 2)
    bwd_small_kernel<2><<<grid, SMALL_THREADS, smem, stream>>>(g, go, w, xt, off, mask, gxt, goff, gmask, gw);
  else if (g.Og <= 4)
    bwd_small_kernel<4><<<grid, SMALL_THREADS, smem, stream>>>(g, go, w, xt, off, mask, gxt, goff, gmask, gw);
  else
    bwd_small_kernel<8><<<grid, SMALL_THREADS, smem, stream>>>(g, go, w, xt, off, mask, gxt, goff, gmask, gw);
  return cudaGetLastError();
}

cudaError_t launch_bwd_weight_simt(const Geom& g, const float* go, const float* xt,
                                   const float* off, const float* mask, float* gw, int num_sms,
                                   cudaStream_t stream) {
  if (g.NP == 0 || g.Cg == 0 || g.Og == 0) return cudaSuccess;
  const long long base = (long long)ceil_div(g.Og, W_BM) * g.kk * ceil_div(g.Cg, W_BN) * g.G;
  long long splits = (4LL * num_sms + base - 1) / base;
  const long long max_splits = (g.NP + 8 * W_BK - 1) / (8 * W_BK);  // >= 8 K steps each
  if (splits > max_splits) splits = max_splits;
  if (splits < 1) splits = 1;
  if (splits * g.G > 65535) splits = 65535 / g.G;
  const long long qps = ((g.NP + splits - 1) / splits + W_BK - 1) / W_BK * W_BK;
  dim3 grid(ceil_div(g.Og, W_BM), g.kk * ceil_div(g.Cg, W_BN), (unsigned)(g.G * splits));
  if (vec8_ok(g))
    bwd_weight_simt_kernel<true><<<grid, 256, 0, stream>>>(g, go, xt, off, mask, gw, (int)splits, qps);
  else
    bwd_weight_simt_kernel<false><<<grid, 256, 0, stream>>>(g, go, xt, off, mask, gw, (int)splits, qps);
  return cudaGetLastError();
}

}  // namespace dcn
