// dcn_dgroup.cu -- forward and backward for small convolution groups that
// tile a deformable group: the channels of one deformable group (cpg of them,
// 4..16) hold GPD whole convolution groups of CG channels and OG out channels
// each -- e.g. groups=32 with 2 channels each and 4 deformable groups: a
// deformable group is 16 channels = 8 convolution groups.
//
// L lanes per (output pixel, deformable group), each with CPG / L channels
// (whole convolution groups, 4 or 8 channels): per tap a lane computes the
// sampling plan (deform_conv2d.metal:100-118) and reads its part of the four
// corner runs of the deformable group's channels with one 16- or 32-byte load
// each from the NHWC input (dropped corners read the zero pixel row after
// it).  The L lanes of a pixel read adjacent runs, so a warp instruction
// covers 32 / L corner runs whole, and every sector fetched is used instead
// of each convolution group re-reading the sector for its few channels.
//  * forward: the OPD = GPD*OG outputs of the pixel, weights in shared memory;
//  * backward: grad columns (K = OG dot products), col2im as 16-byte vector
//    reductions into the NHWC grad-input accumulator, the coordinate and mask
//    gradients of the pixel (summed over its L lanes, stored by the first:
//    plain stores), and its grad_weight products reduced over the warp's
//    pixels with a transpose-reduce and over the block in shared memory.
#include "dcn_kernels.h"

namespace dcn {

namespace {

constexpr int DG_THREADS = 128;

// One run of VW consecutive channels of a corner pixel row: a 256-bit load
// for 8 channels (32-byte aligned: 8 | channels per deformable group), a
// 128-bit load for 4.
template <int VW>
__device__ __forceinline__ void ld_run(const float* p, float (&r)[VW]) {
  if constexpr (VW == 8) {
    asm volatile("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
                 : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]),
                   "=f"(r[6]), "=f"(r[7])
                 : "l"(p));
  } else {
    const float4 v = ldg4(p);
    r[0] = v.x;
    r[1] = v.y;
    r[2] = v.z;
    r[3] = v.w;
  }
}

// Plan of one (pixel, tap, deformable group): element offsets of the four
// corner pixel rows (the zero row for dropped corners), weights, mask.
struct CornerPlan {
  int c[4];
  Sample s;
  float m;
};

__device__ __forceinline__ CornerPlan corner_plan(const Geom& g, const float* __restrict__ off,
                                                  const float* __restrict__ mask, int n, int p,
                                                  int oy, int ox, int k, int dgi) {
  CornerPlan cp;
  const int ki = k / g.kw, kj = k - ki * g.kw;
  const long long oi = off_h_index(g, n, dgi, k, p);
  float h, w;
  sample_pos(g, oy, ox, ki, kj, __ldg(off + oi), __ldg(off + oi + g.P), h, w);
  cp.m = mask_of(g, mask, mask_index(g, n, dgi, k, p));
  cp.s = make_sample(h, w, g.H, g.W);
  const int zoff = g.N * g.HW * g.C;
  const int xn = n * g.HW;
  cp.c[0] = (cp.s.live & 1u) ? (xn + cp.s.i1) * g.C : zoff;
  cp.c[1] = (cp.s.live & 2u) ? (xn + cp.s.i2) * g.C : zoff;
  cp.c[2] = (cp.s.live & 4u) ? (xn + cp.s.i3) * g.C : zoff;
  cp.c[3] = (cp.s.live & 8u) ? (xn + cp.s.i4) * g.C : zoff;
  return cp;
}

template <int CG, int OG, int GPD, int L>
__global__ void __launch_bounds__(DG_THREADS)
fwd_dgroup_kernel(Geom g, const float* __restrict__ xt, const float* __restrict__ w,
                  const float* __restrict__ off, const float* __restrict__ mask,
                  const float* __restrict__ bias, float* __restrict__ out) {
  constexpr int CPG = CG * GPD, OPD = OG * GPD;
  constexpr int CPL = CPG / L, GPL = GPD / L, OPL = GPL * OG;  // per lane
  constexpr int VW = CPL % 8 == 0 ? 8 : 4, NR = CPL / VW;  // channels per load, loads per corner
  static_assert(GPD % L == 0 && CPL % 4 == 0 && 32 % L == 0, "whole groups, 16-byte runs");
  constexpr int NV = OPD * CG, NVL = NV / L;  // weights per tap: of the group, of a lane
  static_assert(NVL % 4 == 0, "16-byte weight loads");
  // the deformable group's weights (out channels dgi*OPD ..), tap-major
  // [kk][OPD][CG], so that a lane's weights of one tap are NVL consecutive floats
  extern __shared__ float ws[];
  const int dgi = blockIdx.y;
  const int wcount = OPD * CG * g.kk;
  for (int i = threadIdx.x; i < wcount; i += DG_THREADS) {
    const int v = i / g.kk;
    ws[(i - v * g.kk) * NV + v] = w[(long long)dgi * wcount + i];
  }
  __syncthreads();
  const int l = threadIdx.x % L;  // this lane's part of the deformable group
  const long long q = ((long long)blockIdx.x * DG_THREADS + threadIdx.x) / L;
  if (q >= g.NP) return;
  const int n = (int)(q / g.P);
  const int p = (int)(q - (long long)n * g.P);
  const int oy = p / g.Wo, ox = p - oy * g.Wo;
  const float* xq = xt + dgi * CPG + l * CPL;
  float acc[OPL];
#pragma unroll
  for (int i = 0; i < OPL; ++i) acc[i] = 0.f;
  for (int k = 0; k < g.kk; ++k) {
    const CornerPlan cp = corner_plan(g, off, mask, n, p, oy, ox, k, dgi);
    if (!cp.s.valid) continue;
    const float w1 = cp.s.w1 * cp.m, w2 = cp.s.w2 * cp.m, w3 = cp.s.w3 * cp.m,
                w4 = cp.s.w4 * cp.m;
    float wk[NVL];  // this lane's weights of tap k: [group][out][channel]
#pragma unroll
    for (int i = 0; i < NVL; i += 4) {
      const float4 t4 = *reinterpret_cast<const float4*>(ws + k * NV + l * NVL + i);
      wk[i] = t4.x;
      wk[i + 1] = t4.y;
      wk[i + 2] = t4.z;
      wk[i + 3] = t4.w;
    }
#pragma unroll
    for (int qd = 0; qd < NR; ++qd) {
      float a[VW], b[VW], c[VW], d[VW];
      ld_run<VW>(xq + (unsigned)cp.c[0] + VW * qd, a);
      ld_run<VW>(xq + (unsigned)cp.c[1] + VW * qd, b);
      ld_run<VW>(xq + (unsigned)cp.c[2] + VW * qd, c);
      ld_run<VW>(xq + (unsigned)cp.c[3] + VW * qd, d);
#pragma unroll
      for (int e = 0; e < VW; ++e) {
        const float v = w1 * a[e] + w2 * b[e] + w3 * c[e] + w4 * d[e];
        const int cl = VW * qd + e;  // channel within this lane's part
        const int j = cl / CG, cc = cl - (cl / CG) * CG;
#pragma unroll
        for (int o = 0; o < OG; ++o)
          acc[j * OG + o] = fmaf(wk[(j * OG + o) * CG + cc], v, acc[j * OG + o]);
      }
    }
  }
#pragma unroll
  for (int i = 0; i < OPL; ++i) {
    const int oc = dgi * OPD + l * OPL + i;
    out[((long long)n * g.outC + oc) * g.P + p] = acc[i] + (g.use_bias ? __ldg(bias + oc) : 0.f);
  }
}

// Sum over the warp's pixels (lanes L apart) of v[0..32/L-1], transposed: the
// lane of pixel slot j (lane / L == j) returns the total of v[j].
template <int L>
__device__ __forceinline__ float pixel_transpose_sum(float (&v)[32 / L], int lane) {
  constexpr int PL = 32 / L;
  int d = 16;
#pragma unroll
  for (int h = PL / 2; h >= 1; h >>= 1, d >>= 1) {
    const bool upper = (lane & d) != 0;
#pragma unroll
    for (int i = 0; i < h; ++i) {
      const float send = upper ? v[i] : v[i + h];
      const float keep = upper ? v[i + h] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
    }
  }
  return v[0];
}

template <int CG, int OG, int GPD, int L>
__global__ void __launch_bounds__(DG_THREADS)
bwd_dgroup_kernel(Geom g, const float* __restrict__ go, const float* __restrict__ w,
                  const float* __restrict__ xt, const float* __restrict__ off,
                  const float* __restrict__ mask, float* __restrict__ gxt,
                  float* __restrict__ goff, float* __restrict__ gmask, float* __restrict__ gw) {
  constexpr int CPG = CG * GPD, OPD = OG * GPD, NV = OPD * CG;
  constexpr int CPL = CPG / L, GPL = GPD / L, OPL = GPL * OG, NVL = NV / L;  // per lane
  constexpr int PL = 32 / L;  // pixels of a warp
  constexpr int VW = CPL % 8 == 0 ? 8 : 4, NR = CPL / VW;  // channels per load, loads per corner
  static_assert(GPD % L == 0 && CPL % 4 == 0 && 32 % L == 0, "whole groups, 16-byte runs");
  static_assert(NVL <= PL, "one grad_weight value per pixel slot of the warp");
  // weights tap-major [kk][OPD][CG] (a lane's weights of one tap: NVL
  // consecutive floats), then the grad_weight sums in the weight's layout
  // [OPD][CG][kk]
  extern __shared__ float sm[];
  const int dgi = blockIdx.y;
  const int wcount = OPD * CG * g.kk;
  float* ws = sm;
  float* gws = sm + wcount;
  for (int i = threadIdx.x; i < wcount; i += DG_THREADS) {
    const int v = i / g.kk;
    ws[(i - v * g.kk) * NV + v] = w[(long long)dgi * wcount + i];
    gws[i] = 0.f;
  }
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int l = lane % L;  // this lane's part of the deformable group
  const long long q = ((long long)blockIdx.x * DG_THREADS + threadIdx.x) / L;
  const bool valid = q < g.NP;  // no early exit: the warp reduces together
  const int n = valid ? (int)(q / g.P) : 0;
  const int p = valid ? (int)(q - (long long)n * g.P) : 0;
  const int oy = p / g.Wo, ox = p - oy * g.Wo;
  float gov[OPL];
#pragma unroll
  for (int i = 0; i < OPL; ++i)
    gov[i] = valid ? __ldg(go + ((long long)n * g.outC + dgi * OPD + l * OPL + i) * g.P + p)
                   : 0.f;
  const float* xq = xt + dgi * CPG + l * CPL;
  float* gq = gxt + dgi * CPG + l * CPL;
  const int zoff = g.N * g.HW * g.C;
  for (int k = 0; k < g.kk; ++k) {
    float gwp[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) gwp[i] = 0.f;
    float s_h = 0.f, s_w = 0.f, s_m = 0.f, mscale = 1.f;
    if (valid) {
      const CornerPlan cp = corner_plan(g, off, mask, n, p, oy, ox, k, dgi);
      mscale = mask_grad_scale(g, cp.m);
      if (cp.s.valid) {
        const float m = cp.m;
        float wk[NVL];  // this lane's weights of tap k: [group][out][channel]
#pragma unroll
        for (int i = 0; i < NVL; i += 4) {
          const float4 t4 = *reinterpret_cast<const float4*>(ws + k * NV + l * NVL + i);
          wk[i] = t4.x;
          wk[i + 1] = t4.y;
          wk[i + 2] = t4.z;
          wk[i + 3] = t4.w;
        }
#pragma unroll
        for (int qd = 0; qd < NR; ++qd) {
          float a[VW], b[VW], c[VW], d[VW];
          ld_run<VW>(xq + (unsigned)cp.c[0] + VW * qd, a);
          ld_run<VW>(xq + (unsigned)cp.c[1] + VW * qd, b);
          ld_run<VW>(xq + (unsigned)cp.c[2] + VW * qd, c);
          ld_run<VW>(xq + (unsigned)cp.c[3] + VW * qd, d);
          float top[VW];
#pragma unroll
          for (int e = 0; e < VW; ++e) {
            const int cl = VW * qd + e;  // channel within this lane's part
            const int j = cl / CG, cc = cl - (cl / CG) * CG;
            float gc = 0.f;  // grad column (.mm:820-821)
#pragma unroll
            for (int o = 0; o < OG; ++o) gc = fmaf(gov[j * OG + o], wk[(j * OG + o) * CG + cc], gc);
            const float A = a[e], B = b[e], Cv = c[e], D = d[e];
            s_h += m * coord_dh(cp.s, A, B, Cv, D) * gc;
            s_w += m * coord_dw(cp.s, A, B, Cv, D) * gc;
            const float val = bilerp(cp.s, A, B, Cv, D);
            s_m += gc * val;
            top[e] = gc * m;
            const float colv = val * m;
#pragma unroll
            for (int o = 0; o < OG; ++o) gwp[(j * OG + o) * CG + cc] = gov[j * OG + o] * colv;
          }
          // col2im (deform_conv2d.metal:141-204): dropped corners are skipped
          const float ws4[4] = {cp.s.w1, cp.s.w2, cp.s.w3, cp.s.w4};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            if (cp.c[i] == zoff) continue;
            const float wi = ws4[i];
#pragma unroll
            for (int h = 0; h < VW; h += 4)
              red_add_v4(gq + (unsigned)cp.c[i] + VW * qd + h, wi * top[h], wi * top[h + 1],
                         wi * top[h + 2], wi * top[h + 3]);
          }
        }
      }
    }
    // the pixel's (deformable group, tap) gradients, summed over its L lanes
    // and stored by the first (col2im_coord, deform_conv2d.metal:225-295)
#pragma unroll
    for (int d = 1; d < L; d <<= 1) {
      s_h += __shfl_xor_sync(0xffffffffu, s_h, d);
      s_w += __shfl_xor_sync(0xffffffffu, s_w, d);
      s_m += __shfl_xor_sync(0xffffffffu, s_m, d);
    }
    if (valid && l == 0) {
      const long long oi = off_h_index(g, n, dgi, k, p);
      goff[oi] = s_h;
      goff[oi + g.P] = s_w;
      if (g.use_mask) gmask[mask_index(g, n, dgi, k, p)] = s_m * mscale;
    }
    const float tot = pixel_transpose_sum<L>(gwp, lane);
    const int jv = lane / L;  // the value this lane now holds
    if (jv < NVL) atomicAdd(&gws[(l * NVL + jv) * g.kk + k], tot);
  }
  __syncthreads();
  for (int i = threadIdx.x; i < wcount; i += DG_THREADS)
    red_add_f32(gw + (long long)dgi * wcount + i, gws[i]);
}

using FwdFn = void (*)(Geom, const float*, const float*, const float*, const float*,
                       const float*, float*);
using BwdFn = void (*)(Geom, const float*, const float*, const float*, const float*,
                       const float*, float*, float*, float*, float*);

struct DgroupEntry {
  int cg, og, gpd, lanes_fwd, lanes_bwd;
  FwdFn fwd;
  BwdFn bwd;
};

#define DG_ENTRY(CG, OG, GPD, LF, LB)                                           \
  {                                                                             \
    CG, OG, GPD, LF, LB, fwd_dgroup_kernel<CG, OG, GPD, LF>,                    \
        bwd_dgroup_kernel<CG, OG, GPD, LB>                                      \
  }

// (channels, out channels) per convolution group x groups per deformable
// group: 4, 8 or 16 channels per deformable group, <= 32 grad_weight values
// per pixel; lanes per (pixel, deformable group): 8 channels each in the
// forward (32-byte loads), 4 in the backward (measured faster on the grouped
// workload: 0.054 / 0.102 ms against 0.060 / 0.140 ms the other way round).
const DgroupEntry kDgroup[] = {
    DG_ENTRY(1, 1, 4, 1, 1),  DG_ENTRY(1, 1, 8, 1, 2), DG_ENTRY(1, 1, 16, 2, 4),
    DG_ENTRY(2, 2, 2, 1, 1),  DG_ENTRY(2, 2, 4, 1, 2), DG_ENTRY(2, 2, 8, 2, 4),
    DG_ENTRY(4, 4, 1, 1, 1),  DG_ENTRY(4, 4, 2, 1, 2), DG_ENTRY(1, 2, 4, 1, 1),
    DG_ENTRY(1, 2, 8, 1, 2),  DG_ENTRY(2, 4, 2, 1, 1), DG_ENTRY(2, 4, 4, 1, 2),
};

const DgroupEntry* find_dgroup(const Geom& g) {
  if (g.cpg % g.Cg != 0 || g.C % 4 != 0) return nullptr;
  const int gpd = g.cpg / g.Cg;
  for (const DgroupEntry& e : kDgroup)
    if (e.cg == g.Cg && e.og == g.Og && e.gpd == gpd) return &e;
  return nullptr;
}

}  // namespace

bool dgroup_supported(const Geom& g) {
  return find_dgroup(g) != nullptr && g.NP > 0 &&
         (long long)g.N * g.HW * g.C + g.C < (1LL << 31) && g.dg <= 65535;
}

cudaError_t launch_fwd_dgroup(const Geom& g, const float* xt, const float* w, const float* off,
                              const float* mask, const float* bias, float* out,
                              cudaStream_t stream) {
  if (!dgroup_supported(g)) return cudaErrorInvalidValue;
  const DgroupEntry* e = find_dgroup(g);
  dim3 grid((unsigned)((g.NP * e->lanes_fwd + DG_THREADS - 1) / DG_THREADS), g.dg);
  const size_t smem = (size_t)g.Og * (g.cpg / g.Cg) * g.Cg * g.kk * sizeof(float);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  e->fwd<<<grid, DG_THREADS, smem, stream>>>(g, xt, w, off, mask, bias, out);
  return cudaGetLastError();
}

cudaError_t launch_bwd_dgroup(const Geom& g, const float* go, const float* w, const float* xt,
                              const float* off, const float* mask, float* gxt, float* goff,
                              float* gmask, float* gw, cudaStream_t stream) {
  if (!dgroup_supported(g)) return cudaErrorInvalidValue;
  const DgroupEntry* e = find_dgroup(g);
  dim3 grid((unsigned)((g.NP * e->lanes_bwd + DG_THREADS - 1) / DG_THREADS), g.dg);
  const size_t smem = 2 * (size_t)g.Og * (g.cpg / g.Cg) * g.Cg * g.kk * sizeof(float);
  if (smem > 48 * 1024) return cudaErrorInvalidValue;
  e->bwd<<<grid, DG_THREADS, smem, stream>>>(g, go, w, xt, off, mask, gxt, goff, gmask, gw);
  return cudaGetLastError();
}

}  // namespace dcn
