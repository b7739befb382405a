// dcn_bwd_tc.cu -- backward deformable convolution on tcgen05 tensor cores
// (kind::tf32, fp32 accumulation in tensor memory).
//
//  prep          go -> go_r (NCHW, rows padded to a multiple of 4 pixels),
//                rounded to TF32 with round-to-nearest (+ the low TF32 parts
//                in 3xTF32), grad_bias summed on the way.
//  bwd_data_tc   per 128-pixel tile of one image and tap k:
//                  gcol[q, c] = sum_o go[q, o] W[o, c, k]            (.mm:820-821)
//                on the tensor core, then an epilogue that reads each pixel's
//                row of gcol out of tensor memory and, in the same pass,
//                  * scatters gcol * mask * corner weight into the NHWC
//                    grad-input accumulator (col2im, deform_conv2d.metal:141-204)
//                    with 16-byte vector reductions;
//                  * sums the coordinate and mask gradients over the channels
//                    (col2im_coord, deform_conv2d.metal:225-295) -- a pixel's
//                    channels are all in its thread, so the sums are local.
//  bwd_weight_tc gW'[c, o] = sum_q col[q, c] go[q, o] for 128 channels of one
//                tap, split over pixel ranges (.mm:842-880).  The column tile
//                is gathered (bilinear sampling, as in the forward) straight
//                into an MN-major operand (32-byte-atom swizzle); go_r rows arrive by
//                cp.async.  Partial tiles are reduced into grad_weight.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "dcn_kernels.h"
#include "dcn_launch.h"
#include "dcn_tc.h"
#include "dcn_tc_common.cuh"
#include "dcn_transpose.cuh"
#include "dcn_tma.h"

namespace dcn {

// Error word of the tensor-core backward: kStatusBwdData / kStatusBwdWeight
// raised by a wait of that kernel that ran out (read and cleared by
// read_bwd_status).
__device__ int g_tc_bwd_status;

namespace {

constexpr int THREADS = 256;

int pow2_cols(int n) {
  int c = 32;
  while (c < n) c <<= 1;
  return c;
}

// ---------------------------------------------------------------------------
// prep: go (N, outC, P) -> go_r (N*outC rows of Ppad), TF32-rounded
// ---------------------------------------------------------------------------
// With `split` (3xTF32) the low TF32 parts fill rows N*outC .. 2*N*outC-1.
// Pixels P .. Ppad-1 of a row are zero.  A block covers PG_SPAN pixels of one
// (image, out channel) row -- 16-byte accesses when P % 4 == 0, all eight of a
// thread's loads issued before their stores -- and, with `gb` (pre-zeroed
// grad_bias), adds its row's sum with one atomic, or with `gpart` writes it
// to gpart[bid] (no atomics; weight_from_tap_major_kernel sums them).  `bid`: the block's
// index among the prep blocks (256 threads).
constexpr int PG_SPAN = 8192;
constexpr int PG_UNROLL = PG_SPAN / (4 * 256);  // float4 loads in flight a thread
__device__ __forceinline__ void prep_go_block(long long bid, const float* __restrict__ go,
                                              float* __restrict__ go_r, float* __restrict__ gb,
                                              float* __restrict__ gpart, int N, int outC, int P,
                                              int Ppad, int pspans, int split, int vec) {
  __shared__ float part[8];
  const long long row = bid / pspans;  // n * outC + o
  const int pbeg = (int)(bid - row * pspans) * PG_SPAN;
  const int pend = min(Ppad, pbeg + PG_SPAN);
  const float* src = go + row * P;
  float* hi = go_r + row * Ppad;
  float* lo = go_r + ((long long)N * outC + row) * Ppad;
  float sum = 0.f;
  if (vec) {  // P % 4 == 0: Ppad == P, 16-byte aligned rows
    float4 v[PG_UNROLL];
#pragma unroll
    for (int u = 0; u < PG_UNROLL; ++u) {
      const int p = pbeg + 4 * (threadIdx.x + u * 256);
      v[u] = p < pend ? __ldg(reinterpret_cast<const float4*>(src + p))
                      : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < PG_UNROLL; ++u) {
      const int p = pbeg + 4 * (threadIdx.x + u * 256);
      if (p >= pend) continue;
      const float4 h = make_float4(tc::to_tf32(v[u].x), tc::to_tf32(v[u].y),
                                   tc::to_tf32(v[u].z), tc::to_tf32(v[u].w));
      *reinterpret_cast<float4*>(hi + p) = h;
      if (split)
        *reinterpret_cast<float4*>(lo + p) =
            make_float4(tc::to_tf32(v[u].x - h.x), tc::to_tf32(v[u].y - h.y),
                        tc::to_tf32(v[u].z - h.z), tc::to_tf32(v[u].w - h.w));
      sum += (v[u].x + v[u].y) + (v[u].z + v[u].w);
    }
  } else {
    for (int p = pbeg + threadIdx.x; p < pend; p += blockDim.x) {
      const float v = p < P ? __ldg(src + p) : 0.f;
      const float h = tc::to_tf32(v);
      hi[p] = h;
      if (split) lo[p] = tc::to_tf32(v - h);
      sum += v;
    }
  }
  if (gb == nullptr && gpart == nullptr) return;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    if (gpart != nullptr) gpart[bid] = t;
    else atomicAdd(gb + row % outC, t);
  }
}
__global__ void __launch_bounds__(256) prep_go_kernel(const float* __restrict__ go,
                                                      float* __restrict__ go_r,
                                                      float* __restrict__ gb, int N, int outC,
                                                      int P, int Ppad, int pspans, int split,
                                                      int vec) {
  prep_go_block(blockIdx.x, go, go_r, gb, nullptr, N, outC, P, Ppad, pspans, split, vec);
}

// MN-major A operands (M contiguous: the channels of the weight gradient's
// columns, the pixels of the grad-column kernel's grad_out).  For 32-bit
// operands the tensor core takes MN-major tiles only in the "128-byte
// swizzle, 32-byte atom" layout: an atom is 4 K rows x 128 B (32 M elements),
// and within it the 32-byte chunk c of row r sits at chunk position c ^ r --
// exactly what TMA writes for a box of 32 elements x K rows with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.  Atoms: K groups of 4 rows at
// W_SBO = 512 B, M blocks of 32 at W_LBO = 4096 B (16 KB per 128 x 32 stage).
constexpr int W_LBO = 4096, W_SBO = 512;

// Instruction descriptor with A MN-major (bit 15), B K-major.
__host__ __device__ constexpr uint32_t idesc_tf32_amn(int M, int N) {
  return tc::idesc_tf32(M, N) | (1u << 15);
}
__device__ __forceinline__ uint64_t sdesc_sw128b32_mn(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(W_LBO >> 4) << 16) |
         ((uint64_t)(W_SBO >> 4) << 32) | (1ull << 46) | (1ull << 61);
}

// ---------------------------------------------------------------------------
// bwd_data_tc
// ---------------------------------------------------------------------------
constexpr int D_BM = 128;
constexpr int D_BN = 128;          // channels of one tap per tile
constexpr int D_TMA_WARP = 0, D_MMA_WARP = 1, D_EPI_WARP0 = 2;
constexpr int D_STAGE = D_BM * 128 + D_BN * 128;             // A + B = 32 KB
// TF32: 3 stages, 16 epilogue warps (4 per tensor-memory lane quarter, 32
// channels each).  3xTF32: the stages carry high and low parts (64 KB), 2
// stages, 8 epilogue warps of 64 channels, to fit shared memory.
template <bool SPLIT> struct DCfg {
  static constexpr int STAGES = SPLIT ? 2 : 3;
  static constexpr int PARTS = SPLIT ? 2 : 1;
  static constexpr int EPI_WARPS = SPLIT ? 8 : 16;
  static constexpr int THREADS = (D_EPI_WARP0 + EPI_WARPS) * 32;
};

// Sampling plan of one pixel for one (tap, deformable group), kept in shared
// memory so that the 8 lanes working on the pixel can read it.
// Four 16-byte words, read with vector loads.
struct __align__(16) PixPlan {
  int4 cidx;       // element offset (n*H*W + y*W + x) * C of each corner; the
                   // zero row for dropped corners
  float4 w;        // bilinear weights (0 for dropped corners)
  float4 geo;      // lh, lw (fractional position), msk (modulation), unused
  int4 idx;        // offset-gradient index of (n, dgi, k, p) (-1: pixel or
                   // sample void), mask-gradient index, unused x2
};
static_assert(sizeof(PixPlan) == 64, "PixPlan is 4 x 16 bytes");

constexpr int EPI_TSTRIDE = 36;  // transpose buffer row stride (floats): 16-byte rows
constexpr int EPI_T_BYTES = 32 * EPI_TSTRIDE * 4;  // 4608: keeps the plans 16-byte aligned
constexpr int EPI_WARP_BYTES = EPI_T_BYTES + 32 * (int)sizeof(PixPlan);  // 6656

size_t data_smem_bytes(bool split) {
  const int stages = split ? DCfg<true>::STAGES : DCfg<false>::STAGES;
  const int parts = split ? 2 : 1;
  const int epi = split ? DCfg<true>::EPI_WARPS : DCfg<false>::EPI_WARPS;
  return (size_t)stages * parts * D_STAGE + (size_t)epi * EPI_WARP_BYTES + 128 + 1024;
}

// The packed weight of a group is kk*Cg rows ordered (tap, channel); a
// "slot" is 128 consecutive rows of it: 128 channels of one tap when
// Cg % 128 == 0, or 128 / Cg whole taps when Cg is 32 or 64 (the last slot
// of a group may reach past its last tap; those columns are not used).  A
// tile is (128 pixels, group, range of slots); slots are independent here,
// so splitting them evens out the CTAs' loads.  The pixel side counts
// 32-pixel blocks of one image each (`bpi` per image, the last one partial):
// a tile is 4 consecutive blocks, one per tensor-memory lane quarter, and
// each block's grad_out rows come from its own image.
struct DTile {
  int b0;  // first 32-pixel block
  int gi, s0, s1;
};
__device__ __forceinline__ DTile dtile_of(int t, int mtiles, int nslots, int ksplits) {
  DTile T;
  const int ks = t % ksplits;
  const int r = t / ksplits;
  T.b0 = (r % mtiles) * 4;
  T.gi = r / mtiles;
  T.s0 = ks * nslots / ksplits;
  T.s1 = (ks + 1) * nslots / ksplits;
  return T;
}

// Streaming (evict-first) 32-byte global store (sm_100: 256-bit vectors).
__device__ __forceinline__ void st_cs_v8(float* p, const float (&v)[8]) {
  asm volatile("st.global.cs.v8.f32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p),
               "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]),
               "f"(v[7])
               : "memory");
}
// 32-byte read-only global load (sm_100), 32-byte aligned.  Not volatile: the
// input copy is not written while the kernel runs, so the loads may be
// scheduled freely.
__device__ __forceinline__ void ldg_f8(const float* p, float (&r)[8]) {
  asm("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=f"(r[0]), "=f"(r[1]), "=f"(r[2]), "=f"(r[3]), "=f"(r[4]), "=f"(r[5]), "=f"(r[6]),
        "=f"(r[7])
      : "l"(p));
}

// Predicated vector / scalar reductions: no branch around the instruction.
__device__ __forceinline__ void red_add_v4_if(bool p, float* addr, float a, float b, float c,
                                              float d) {
  asm volatile(
      "{\n.reg .pred q;\nsetp.ne.b32 q, %5, 0;\n"
      "@q red.global.add.v4.f32 [%0], {%1, %2, %3, %4};\n}\n" ::"l"(addr),
      "f"(a), "f"(b), "f"(c), "f"(d), "r"((int)p)
      : "memory");
}
__device__ __forceinline__ void red_add_f32_if(bool p, float* addr, float a) {
  asm volatile("{\n.reg .pred q;\nsetp.ne.b32 q, %2, 0;\n@q red.global.add.f32 [%0], %1;\n}\n" ::"l"(
                   addr),
               "f"(a), "r"((int)p)
               : "memory");
}

// One epilogue warp, one tap: 32 pixel rows x 32 channels of the grad-column
// accumulator.  Tensor memory gives each lane its own pixel's row; the rows go
// through a shared-memory transpose (rows 36 floats apart: every access
// below is free of bank conflicts within a quarter warp).  The gather runs 4
// lanes to a pixel, 8 channels each, so that every corner load is one 32-byte
// vector and a warp instruction covers 8 pixels; the scatter into the NHWC
// grad-input accumulator (col2im) runs 8 lanes to a pixel, 4 channels each,
// so that every quarter warp's 16-byte vector reductions fill one 128-byte
// line (the L1 handles reductions one line per quarter warp at best).  Each
// lane keeps its gather pixel's sampling plan in registers, and the pixel
// pair a quarter warp reduces is the pair of lanes L and L ^ 4, so the
// scatter takes the plans by shuffle.  The coordinate / mask gradients of each
// pixel are reduced over its channels.  With a column buffer (`col` non-NULL)
// it also stores the sampled column values col[k][q][c] = mask * bilinear(x)
// -- TF32-rounded; with `col_lo` non-zero the low TF32 parts go `col_lo`
// floats further -- for the weight gradient.
//
// The coordinate and mask gradients need, per pixel, only the four sums
// D_i = sum_c gcol[c] * v_i[c] over the channels of the corner values v_i:
//   d/dh = m ((1 - lw) (D3 - D1) + lw (D4 - D2))
//   d/dw = m ((1 - lh) (D2 - D1) + lh (D4 - D3))
//   d/dm = w1 D1 + w2 D2 + w3 D3 + w4 D4
// (bilinear.metalh:73-99 per channel, summed over the channels by
// deform_conv2d.metal:225-295), so a lane accumulates four products per
// channel and the pixel's lanes combine the sums once.
__device__ __forceinline__ void epilogue_chunk(const Geom& g, int k, const float (&vals)[32],
                                               int gch0, long long row_q, long long qbase,
                                               int lane, unsigned char* scratch,
                                               const float* __restrict__ xt,
                                               const float* __restrict__ off,
                                               const float* __restrict__ mask,
                                               float* __restrict__ gxt, float* __restrict__ goff,
                                               float* __restrict__ gmask, float* __restrict__ col,
                                               long long col_lo, long long qend, int& plan_key) {
  float* T = reinterpret_cast<float*>(scratch);
  PixPlan* plan = reinterpret_cast<PixPlan*>(scratch + EPI_T_BYTES);
  const int quad = lane & 3, sub = lane >> 2;
  const int zoff = g.N * g.HW * g.C;
  const int dgi = gch0 / g.cpg;
  const int key = k * 65536 + dgi;
  __syncwarp();
  if (key != plan_key) {
    plan_key = key;
    int4 cidx = make_int4(zoff, zoff, zoff, zoff);
    float4 wv4 = make_float4(0.f, 0.f, 0.f, 0.f);
    float4 geo = make_float4(0.f, 0.f, 0.f, 0.f);
    int4 idx = make_int4(-1, 0, 0, 0);
    if (row_q < qend) {
      const int n = (int)(row_q / g.P);
      const int p = (int)(row_q - (long long)n * g.P);
      const int oy = p / g.Wo, ox = p - oy * g.Wo;
      const int ki = k / g.kw, kj = k - ki * g.kw;
      const long long oi = off_h_index(g, n, dgi, k, p);
      float h, w;
      sample_pos(g, oy, ox, ki, kj, __ldg(off + oi), __ldg(off + oi + g.P), h, w);
      const Sample sp = make_sample(h, w, g.H, g.W);
      if (sp.valid) {
        const int nb = n * g.HW;
        cidx.x = (sp.live & 1u) ? (nb + sp.i1) * g.C : zoff;
        cidx.y = (sp.live & 2u) ? (nb + sp.i2) * g.C : zoff;
        cidx.z = (sp.live & 4u) ? (nb + sp.i3) * g.C : zoff;
        cidx.w = (sp.live & 8u) ? (nb + sp.i4) * g.C : zoff;
        wv4 = make_float4(sp.w1, sp.w2, sp.w3, sp.w4);
        geo.x = sp.lh;
        geo.y = sp.lw;
        geo.z = mask_of(g, mask, mask_index(g, n, dgi, k, p));
        idx.x = (int)oi;
        idx.y = (int)mask_index(g, n, dgi, k, p);
      }
    }
    PixPlan pl;
    pl.cidx = cidx;
    pl.w = wv4;
    pl.geo = geo;
    pl.idx = idx;
    plan[lane] = pl;
  }
  {  // this lane's pixel row, 16 bytes at a time
    float4* trow = reinterpret_cast<float4*>(T + lane * EPI_TSTRIDE);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      trow[j] = make_float4(vals[4 * j], vals[4 * j + 1], vals[4 * j + 2], vals[4 * j + 3]);
  }
  __syncwarp();
  const float* xq = xt + gch0 + quad * 8;  // corner loads: channels 8 quad .. 8 quad + 7
#pragma unroll 2
  for (int i = 0; i < 4; ++i) {
    const int px = i * 8 + sub;
    const PixPlan pl = plan[px];
    const bool live = pl.idx.x >= 0;
    const float m = pl.geo.z;
    // corner weights times the mask (0 for void samples)
    const float mw[4] = {m * pl.w.x, m * pl.w.y, m * pl.w.z, m * pl.w.w};
    float d1 = 0.f, d2 = 0.f, d3 = 0.f, d4 = 0.f;
    float cv[8];  // column values (mask * bilinear)
#pragma unroll
    for (int e = 0; e < 8; ++e) cv[e] = 0.f;
    if (live) {
      const float* trow = T + px * EPI_TSTRIDE;
      const float4 ga = *reinterpret_cast<const float4*>(trow + quad * 8);
      const float4 gb = *reinterpret_cast<const float4*>(trow + quad * 8 + 4);
      const float gc[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
      float a[8], b[8], c[8], d[8];
      ldg_f8(xq + (unsigned)pl.cidx.x, a);  // dropped corners: zero row
      ldg_f8(xq + (unsigned)pl.cidx.y, b);
      ldg_f8(xq + (unsigned)pl.cidx.z, c);
      ldg_f8(xq + (unsigned)pl.cidx.w, d);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d1 = fmaf(gc[e], a[e], d1);
        d2 = fmaf(gc[e], b[e], d2);
        d3 = fmaf(gc[e], c[e], d3);
        d4 = fmaf(gc[e], d[e], d4);
        cv[e] = mw[0] * a[e] + mw[1] * b[e] + mw[2] * c[e] + mw[3] * d[e];
      }
    }
    if (col != nullptr && qbase + px < qend) {  // every (k, q, c) is written, voids as 0
      float* dst = col + ((long long)k * g.NP + qbase + px) * g.C + gch0 + quad * 8;
      float hi[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) hi[e] = tc::to_tf32(cv[e]);
      // evict-first: the 280 MB of columns must not push the input and the
      // grad-input accumulator (re-read and reduced here) out of L2
      st_cs_v8(dst, hi);
      if (col_lo != 0) {
        float lo[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) lo[e] = tc::to_tf32(cv[e] - hi[e]);
        st_cs_v8(dst + col_lo, lo);
      }
    }
    // the four sums over the pixel's 4 lanes; lanes 0, 1, 2 of the pixel
    // reduce d/dh, d/dw, d/dm into memory
    d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
    d2 += __shfl_xor_sync(0xffffffffu, d2, 1);
    d3 += __shfl_xor_sync(0xffffffffu, d3, 1);
    d4 += __shfl_xor_sync(0xffffffffu, d4, 1);
    d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
    d2 += __shfl_xor_sync(0xffffffffu, d2, 2);
    d3 += __shfl_xor_sync(0xffffffffu, d3, 2);
    d4 += __shfl_xor_sync(0xffffffffu, d4, 2);
    {  // lane quad 0: d/dh, 1: d/dw, 2: d/dm (mask), 3: nothing
      const float dh = m * ((1.f - pl.geo.y) * (d3 - d1) + pl.geo.y * (d4 - d2));
      const float dw = m * ((1.f - pl.geo.x) * (d2 - d1) + pl.geo.x * (d4 - d3));
      const float dm = (pl.w.x * d1 + pl.w.y * d2 + pl.w.z * d3 + pl.w.w * d4) *
                       mask_grad_scale(g, m);
      const float v = quad == 0 ? dh : (quad == 1 ? dw : dm);
      // void samples carry idx.x = -1: the address is not formed for them
      float* dst = quad == 2 ? gmask + (live ? pl.idx.y : 0)
                             : goff + (live ? pl.idx.x : 0) + (quad == 1 ? g.P : 0);
      red_add_f32_if(live && quad < (g.use_mask ? 3 : 2), dst, v);
    }
    // col2im: 8 lanes per pixel, 4 channels each, so that each quarter warp's
    // 16-byte reductions fill one pixel's 128-byte line.  Lanes L and L ^ 4
    // hold the plans of the pixel pair (i * 8 + 2 (sub / 2), + 1) that lanes
    // L & ~7 .. L | 7 reduce.
    const int oc[4] = {__shfl_xor_sync(0xffffffffu, pl.cidx.x, 4),
                       __shfl_xor_sync(0xffffffffu, pl.cidx.y, 4),
                       __shfl_xor_sync(0xffffffffu, pl.cidx.z, 4),
                       __shfl_xor_sync(0xffffffffu, pl.cidx.w, 4)};
    const float omw[4] = {__shfl_xor_sync(0xffffffffu, mw[0], 4),
                          __shfl_xor_sync(0xffffffffu, mw[1], 4),
                          __shfl_xor_sync(0xffffffffu, mw[2], 4),
                          __shfl_xor_sync(0xffffffffu, mw[3], 4)};
    const bool olive = __shfl_xor_sync(0xffffffffu, (int)live, 4) != 0;
    const int j = lane & 7;
    float* gq = gxt + gch0 + j * 4;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const bool own = h == (sub & 1);
      const bool hl = own ? live : olive;
      const int rp = i * 8 + (sub & ~1) + h;
      const float4 g4 = *reinterpret_cast<const float4*>(T + rp * EPI_TSTRIDE + j * 4);
      const int cis[4] = {own ? pl.cidx.x : oc[0], own ? pl.cidx.y : oc[1],
                          own ? pl.cidx.z : oc[2], own ? pl.cidx.w : oc[3]};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        // dropped corners (the zero row) and void samples are not reduced
        const bool on = hl && cis[cc] != zoff;
        const float wc = own ? mw[cc] : omw[cc];
        red_add_v4_if(on, gq + (unsigned)(on ? cis[cc] : 0), wc * g4.x, wc * g4.y, wc * g4.z,
                      wc * g4.w);
      }
    }
  }
}

// Persistent, warp-specialised grad-column kernel.  Tile = four 32-pixel
// blocks (128 pixels) x one 128-row slot of a group's (tap, channel) rows;
// per slot a K = Og GEMM into one of two tensor-memory accumulators (slots
// alternate), consumed by 16 epilogue warps while the next slot accumulates.
//   warp 0      TMA producer per K step: for each pixel block, 32 out channels
//               x 32 pixels of its image's go_r rows (an MN-major operand),
//               and packed weight rows (128 channels x 32 out channels)
//   warp 1      MMA issue: 4 UMMAs 128 x 128 x 8 per K step
//   warps 2-17  epilogue (epilogue_chunk)
template <bool SPLIT>
__global__ void __launch_bounds__(DCfg<SPLIT>::THREADS, 1)
bwd_data_tc_kernel(Geom g, const __grid_constant__ CUtensorMap amap,
                   const __grid_constant__ CUtensorMap bmap, int bpi, int nblocks, int mtiles,
                   int nslots, int ksplits, int ntiles,
                   const float* __restrict__ xt, const float* __restrict__ off,
                   const float* __restrict__ mask, float* __restrict__ gxt,
                   float* __restrict__ goff, float* __restrict__ gmask,
                   float* __restrict__ col) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw_u32 & 1023u)) & 1023u);
  constexpr int D_STAGES = DCfg<SPLIT>::STAGES;
  constexpr int PARTS = DCfg<SPLIT>::PARTS;
  constexpr int D_EPI_WARPS = DCfg<SPLIT>::EPI_WARPS;
  constexpr int SSTAGE = PARTS * D_STAGE;  // [A_hi B_hi] ([A_lo B_lo])
  const uint32_t s0 = tc::smem_u32(smem);
  unsigned char* epi = smem + D_STAGES * SSTAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(epi + D_EPI_WARPS * EPI_WARP_BYTES);
  uint64_t* empty = full + D_STAGES;
  uint64_t* acc_full = empty + D_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const tc::Watch watch{abort_flag, &g_tc_bwd_status, kStatusBwdData, g.wait_limit};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 32-out-channel K steps; a partial last one reads zero weights past Og
  // (the weight map ends there), so the grad_out rows it also loads add nothing
  const int ochunks = (g.Og + 31) >> 5;

  if (tid == 0) {
    for (int s = 0; s < D_STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&acc_full[a], 1);
      tc::mbar_init(&acc_empty[a], D_EPI_WARPS);
    }
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == D_MMA_WARP) {
    tc::tmem_alloc(tmem_slot, 2 * D_BN);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == D_TMA_WARP) {
    if (lane == 0 && !g.no_async) {
      int gs = 0;  // stages filled so far
      [&]() {
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const DTile T = dtile_of(t, mtiles, nslots, ksplits);
        // per block: go_r row of out channel 0 of its image, first pixel; a
        // block past the last image loads past the row end (zero fill)
        int arow[4], ax[4];
#pragma unroll
        for (int mb = 0; mb < 4; ++mb) {
          const int b = T.b0 + mb;
          const int n = b < nblocks ? b / bpi : 0;
          arow[mb] = n * g.outC + T.gi * g.Og;
          ax[mb] = b < nblocks ? (b - n * bpi) * 32 : bpi * 32;
        }
        for (int sl = T.s0; sl < T.s1; ++sl) {
          const int brow = T.gi * g.kk * g.Cg + sl * D_BN;
          for (int s = 0; s < ochunks; ++s, ++gs) {
            const int st = gs % D_STAGES;
            const int u = gs / D_STAGES;
            if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return;
            tc::mbar_arrive_expect_tx(&full[st], SSTAGE);
            const uint32_t sA = s0 + st * SSTAGE;
            // pixels past the image's last one are outside the map: zero fill
#pragma unroll
            for (int mb = 0; mb < 4; ++mb)
              tc::tma_load_2d(sA + mb * W_LBO, &amap, ax[mb], arow[mb] + s * 32, &full[st]);
            tc::tma_load_2d(sA + D_BM * 128, &bmap, s * 32, brow, &full[st]);
            if constexpr (SPLIT) {  // low parts: rows N*outC further
#pragma unroll
              for (int mb = 0; mb < 4; ++mb)
                tc::tma_load_2d(sA + D_STAGE + mb * W_LBO, &amap, ax[mb],
                                g.N * g.outC + arow[mb] + s * 32, &full[st]);
              tc::tma_load_2d(sA + D_STAGE + D_BM * 128, &bmap, s * 32, g.G * g.kk * g.Cg + brow,
                              &full[st]);
            }
          }
        }
      }
      }();
      if (tc::aborted(watch))  // the copies of the last stages land before exit
        for (int i = gs > D_STAGES ? gs - D_STAGES : 0; i < gs; ++i)
          tc::drain_wait(&full[i % D_STAGES], (i / D_STAGES) & 1, g.wait_limit);
    }
    __syncwarp();
  } else if (warp == D_MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32_amn(D_BM, D_BN);
      int gs = 0, gt = 0;
      [&]() {
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const DTile T = dtile_of(t, mtiles, nslots, ksplits);
        for (int sl = T.s0; sl < T.s1; ++sl, ++gt) {
          const int acc = gt & 1;
          if (gt >= 2 && !tc::wait(watch, &acc_empty[acc], ((gt >> 1) - 1) & 1)) return;
          tc::tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(acc * D_BN);
          for (int s = 0; s < ochunks; ++s, ++gs) {
            const int st = gs % D_STAGES;
            if (!tc::wait(watch, &full[st], (gs / D_STAGES) & 1)) return;
            tc::tc_fence_after();
            const uint32_t sA = s0 + st * SSTAGE, sB = sA + D_BM * 128;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              // A: MN-major, K rows j * 8 .. j * 8 + 7 of the stage
              if constexpr (SPLIT) {  // lo x hi + hi x lo + hi x hi
                tc::umma_tf32(d, sdesc_sw128b32_mn(sA + D_STAGE + j * 2 * W_SBO),
                              tc::sdesc_sw128(sB + j * 32), idesc, (s | j) != 0 ? 1u : 0u);
                tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                              tc::sdesc_sw128(sB + D_STAGE + j * 32), idesc, 1u);
                tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                              tc::sdesc_sw128(sB + j * 32), idesc, 1u);
              } else {
                tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                              tc::sdesc_sw128(sB + j * 32), idesc, (s | j) != 0 ? 1u : 0u);
              }
            }
            tc::umma_commit(&empty[st]);
          }
          tc::umma_commit(&acc_full[acc]);
        }
      }
      }();
      if (tc::aborted(watch)) {  // every UMMA issued so far completes before exit
        tc::umma_commit(drain);
        tc::drain_wait(drain, 0, g.wait_limit);
      }
    }
    __syncwarp();
  } else {
    const int e = warp - D_EPI_WARP0;
    const int lq = warp & 3;      // tensor-memory lane quarter this warp may read
    constexpr int CPW = 16 / D_EPI_WARPS;  // 32-channel chunks per warp
    unsigned char* scratch = epi + e * EPI_WARP_BYTES;
    int gt = 0;
    [&]() {
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const DTile T = dtile_of(t, mtiles, nslots, ksplits);
      // this lane quarter's block: pixels qbase .. qbase + 31 of the flat
      // (image, pixel) index, valid below qend (0 for a block past the end)
      const int blk = T.b0 + lq;
      const int bn_ = blk < nblocks ? blk / bpi : 0;
      const long long qbase =
          blk < nblocks ? (long long)bn_ * g.P + (long long)(blk - bn_ * bpi) * 32 : 0;
      const long long qend = blk < nblocks ? (long long)bn_ * g.P + g.P : 0;
      const long long row_q = qbase + lane;
      const long long col_lo = SPLIT ? (long long)g.kk * g.NP * g.C : 0;
      int plan_key = -1;
      for (int sl = T.s0; sl < T.s1; ++sl, ++gt) {
        const int acc = gt & 1;
        if (!tc::wait(watch, &acc_full[acc], (gt >> 1) & 1)) return;
        tc::tc_fence_after();
#pragma unroll 1
        for (int cc = 0; cc < CPW; ++cc) {
          const int chunk = (e >> 2) * CPW + cc;  // 32-channel chunk of the tile
          float vals[32];
          {
            const uint32_t ta =
                tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(acc * D_BN + chunk * 32);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float tv[8];
              tc::tmem_ld8(ta + 8 * j, tv);
#pragma unroll
              for (int q = 0; q < 8; ++q) vals[8 * j + q] = tv[q];
            }
            tc::tmem_ld_wait();
          }
          if (cc == CPW - 1) {
            tc::tc_fence_before();
            __syncwarp();
            if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);  // accumulator free for slot + 2
          }
          const int row = sl * D_BN + chunk * 32;  // (tap, channel) row within the group
          const int k = row / g.Cg;
          if (k < g.kk)
            epilogue_chunk(g, k, vals, T.gi * g.Cg + (row - k * g.Cg), row_q, qbase, lane,
                           scratch, xt, off, mask, gxt, goff, gmask, col, col_lo, qend,
                           plan_key);
        }
      }
    }
    }();
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == D_MMA_WARP) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 2 * D_BN);
  }
}

// ---------------------------------------------------------------------------
// sampling plans: one 32-byte record per (n, deformable group, tap, pixel):
// the element offsets ((n*H*W + y*W + x) * C) of the four corners -- the zero
// row for dropped corners -- and their bilinear weights times the mask.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) plan_kernel(Geom g, const float* __restrict__ off,
                                                   const float* __restrict__ mask,
                                                   int4* __restrict__ plans) {
  const long long total = (long long)g.N * g.dg * g.kk * g.P;
  const int zoff = g.N * g.HW * g.C;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(i % g.P);
    long long r = i / g.P;
    const int k = (int)(r % g.kk);
    r /= g.kk;
    const int dgi = (int)(r % g.dg);
    const int n = (int)(r / g.dg);
    const int oy = p / g.Wo, ox = p - oy * g.Wo;
    const int ki = k / g.kw, kj = k - ki * g.kw;
    const long long oi = off_h_index(g, n, dgi, k, p);
    float h, w;
    sample_pos(g, oy, ox, ki, kj, __ldg(off + oi), __ldg(off + oi + g.P), h, w);
    const float m = mask_of(g, mask, mask_index(g, n, dgi, k, p));
    const Sample sp = make_sample(h, w, g.H, g.W);
    int4 o = make_int4(zoff, zoff, zoff, zoff);
    float4 wv = make_float4(0.f, 0.f, 0.f, 0.f);
    if (sp.valid) {
      const int nb = n * g.HW;
      if (sp.live & 1u) { o.x = (nb + sp.i1) * g.C; wv.x = sp.w1 * m; }
      if (sp.live & 2u) { o.y = (nb + sp.i2) * g.C; wv.y = sp.w2 * m; }
      if (sp.live & 4u) { o.z = (nb + sp.i3) * g.C; wv.z = sp.w3 * m; }
      if (sp.live & 8u) { o.w = (nb + sp.i4) * g.C; wv.w = sp.w4 * m; }
    }
    plans[2 * i] = o;
    plans[2 * i + 1] = make_int4(__float_as_int(wv.x), __float_as_int(wv.y),
                                 __float_as_int(wv.z), __float_as_int(wv.w));
  }
}

// ---------------------------------------------------------------------------
// bwd_weight_tc
// ---------------------------------------------------------------------------
constexpr int W_BM = 128;  // channels of one tap per CTA
// Byte offset of channel quad `quad` (channels 4*quad .. 4*quad+3 of a
// 32-channel block) of pixel `pix` (0..31 of the stage) in one channel block.
__device__ __forceinline__ uint32_t mn32_offset(int pix, int quad) {
  const int kr = pix & 3;
  return (uint32_t)((pix >> 2) * W_SBO + kr * 128 + ((((quad >> 1) ^ kr) & 3) << 5) +
                    ((quad & 1) << 4));
}

// Persistent, warp-specialised weight-gradient kernel.  A tile is (tap k,
// 128 input channels, bn out channels, group, pixel range); its K loop runs
// over 32-pixel chunks of the range.
//   warps 0-3   epilogue: accumulator -> fp32 reductions into grad_weight
//   warp  4     MMA issue: 4 UMMAs 128(channels) x bn x 8(pixels) per K step
//   warp  5     TMA producer of go_r rows (bn out channels x 32 pixels)
//   warps 6-21  16 gather warps: 32 channels x 8 pixels each; the column
//               values are written MN-major (channels contiguous).
// Stage ring and accumulator double buffering as in the forward kernel.
constexpr int W2_GATHER_WARPS = 16;
constexpr int W2_MMA_WARP = 4, W2_TMA_WARP = 5, W2_GATHER_WARP0 = 6;
constexpr int W2_THREADS = (W2_GATHER_WARP0 + W2_GATHER_WARPS) * 32;  // 704
constexpr int W2_A_STAGE = 16384;

// 3xTF32 carries high and low parts: 2 stages of twice the size.
size_t weight_smem_bytes(int bn, bool split) {
  const int stages = split ? 2 : 4, parts = split ? 2 : 1;
  return (size_t)stages * parts * (W2_A_STAGE + (size_t)bn * 128) + 256 + 1024;
}

struct WTile {
  int k, cm0, o0, gi, t_begin, t_end;
};
__device__ __forceinline__ WTile wtile_of(const Geom& g, int t, int mtiles, int ntn, int splits,
                                          int per, int total_chunks, int bn) {
  WTile T;
  const int sp = t % splits;
  int r = t / splits;
  const int nt = r % ntn;
  r /= ntn;
  const int mt = r % mtiles;
  r /= mtiles;
  T.k = r % g.kk;
  T.gi = r / g.kk;
  T.cm0 = mt * W_BM;
  T.o0 = nt * bn;
  T.t_begin = sp * per;
  T.t_end = min(total_chunks, T.t_begin + per);
  return T;
}

template <bool SPLIT>
__global__ void __launch_bounds__(W2_THREADS, 1)
bwd_weight_tc_kernel(Geom g, const __grid_constant__ CUtensorMap gomap, int bn, int tcols,
                     const float* __restrict__ xt, const int4* __restrict__ plans,
                     float* __restrict__ gw, int sk, int sc, int mtiles, int ntn, int splits,
                     int per, int ntiles) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw_u32 & 1023u)) & 1023u);
  constexpr int W2_STAGES = SPLIT ? 2 : 4;
  constexpr int PARTS = SPLIT ? 2 : 1;
  const uint32_t sA0 = tc::smem_u32(smem);
  const uint32_t b_stage = (uint32_t)bn * 128;
  const uint32_t sB0 = sA0 + W2_STAGES * PARTS * W2_A_STAGE;
  uint64_t* full =
      reinterpret_cast<uint64_t*>(smem + W2_STAGES * PARTS * (W2_A_STAGE + b_stage));
  uint64_t* tfull = full + W2_STAGES;  // the go_r rows' TMA bytes
  uint64_t* empty = tfull + W2_STAGES;
  uint64_t* acc_full = empty + W2_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const tc::Watch watch{abort_flag, &g_tc_bwd_status, kStatusBwdWeight, g.wait_limit};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pchunks = (g.P + 31) >> 5;
  const int total_chunks = g.N * pchunks;

  if (tid == 0) {
    for (int s = 0; s < W2_STAGES; ++s) {
      tc::mbar_init(&full[s], W2_GATHER_WARPS);
      tc::mbar_init(&tfull[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&acc_full[a], 1);
      tc::mbar_init(&acc_empty[a], 4);
    }
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == W2_MMA_WARP) {
    tc::tmem_alloc(tmem_slot, (uint32_t)tcols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= W2_GATHER_WARP0) {
    // ------------------------------ gather ------------------------------
    const int gwp = warp - W2_GATHER_WARP0;
    const int mb = gwp & 3, pg = gwp >> 2;
    const int quad = lane & 7, sub = lane >> 3;
    const int zoff = g.N * g.HW * g.C;
    int gs = 0;
    [&]() {
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const WTile T = wtile_of(g, t, mtiles, ntn, splits, per, total_chunks, bn);
      if (T.t_begin >= T.t_end) continue;
      const int gch = T.gi * g.Cg + T.cm0 + mb * 32 + quad * 4;
      const int dgi = (T.gi * g.Cg + T.cm0 + mb * 32) / g.cpg;
      const float* xq = xt + gch;
      uint32_t soff[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) soff[i] = mb * W_LBO + mn32_offset(pg * 8 + i * 4 + sub, quad);
      // The sampling plans of the next K step are loaded one step ahead, so
      // each step waits for one L2 round trip (its corners).
      const int4* plan_k = plans + 2 * ((long long)dgi * g.kk + T.k) * g.P;  // + n*dg*kk*P
      const long long plan_n_stride = 2LL * g.dg * g.kk * g.P;
      int n = T.t_begin / pchunks;
      int p0 = (T.t_begin - n * pchunks) << 5;
      int4 npo[2], npw[2];
      auto fetch = [&](int fn, int fp0) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int pp = fp0 + pg * 8 + i * 4 + sub;
          if (pp < g.P && fn < g.N) {
            const int4* rec = plan_k + fn * plan_n_stride + 2 * pp;
            npo[i] = __ldg(rec);
            npw[i] = __ldg(rec + 1);
          } else {
            npo[i] = make_int4(zoff, zoff, zoff, zoff);
            npw[i] = make_int4(0, 0, 0, 0);
          }
        }
      };
      fetch(n, p0);
      for (int tt = T.t_begin; tt < T.t_end; ++tt, ++gs) {
        const int st = gs % W2_STAGES;
        const int u = gs / W2_STAGES;
        const int coff[2][4] = {{npo[0].x, npo[0].y, npo[0].z, npo[0].w},
                                {npo[1].x, npo[1].y, npo[1].z, npo[1].w}};
        const float cw[2][4] = {{__int_as_float(npw[0].x), __int_as_float(npw[0].y),
                                 __int_as_float(npw[0].z), __int_as_float(npw[0].w)},
                                {__int_as_float(npw[1].x), __int_as_float(npw[1].y),
                                 __int_as_float(npw[1].z), __int_as_float(npw[1].w)}};
        p0 += 32;
        if (p0 >= g.P) {
          p0 = 0;
          ++n;
        }
        float4 v[2][4];
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
          for (int c = 0; c < 4; ++c)
            v[i][c] = ldg4(xq + (unsigned)coff[i][c]);  // dropped corners: zero row
        if (tt + 1 < T.t_end) fetch(n, p0);
        if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return;
        const uint32_t sA = sA0 + st * PARTS * W2_A_STAGE;
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const float a = cw[i][0], b = cw[i][1], c = cw[i][2], d = cw[i][3];
          const float4 A = v[i][0], B = v[i][1], C = v[i][2], D = v[i][3];
          const float e0 = a * A.x + b * B.x + c * C.x + d * D.x;
          const float e1 = a * A.y + b * B.y + c * C.y + d * D.y;
          const float e2 = a * A.z + b * B.z + c * C.z + d * D.z;
          const float e3 = a * A.w + b * B.w + c * C.w + d * D.w;
          const float h0 = tc::to_tf32(e0), h1 = tc::to_tf32(e1), h2 = tc::to_tf32(e2),
                      h3 = tc::to_tf32(e3);
          tc::st_shared_v4(sA + soff[i], h0, h1, h2, h3);
          if constexpr (SPLIT)
            tc::st_shared_v4(sA + W2_A_STAGE + soff[i], tc::to_tf32(e0 - h0), tc::to_tf32(e1 - h1),
                             tc::to_tf32(e2 - h2), tc::to_tf32(e3 - h3));
        }
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&full[st]);
      }
    }
    }();
  } else if (warp == W2_TMA_WARP) {
    // ------------------------------ go_r rows (TMA) ------------------------------
    if (lane == 0 && !g.no_async) {
      int gs = 0;  // stages filled so far
      [&]() {
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const WTile T = wtile_of(g, t, mtiles, ntn, splits, per, total_chunks, bn);
        for (int tt = T.t_begin; tt < T.t_end; ++tt, ++gs) {
          const int st = gs % W2_STAGES;
          const int u = gs / W2_STAGES;
          const int n = tt / pchunks;
          const int p0 = (tt - n * pchunks) << 5;
          if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return;
          tc::mbar_arrive_expect_tx(&tfull[st], PARTS * b_stage);
          const int row = n * g.outC + T.gi * g.Og + T.o0;
          const uint32_t sB = sB0 + st * PARTS * b_stage;
          tc::tma_load_2d(sB, &gomap, p0, row, &tfull[st]);
          if constexpr (SPLIT)  // low parts: rows N*outC .. of go_r
            tc::tma_load_2d(sB + b_stage, &gomap, p0, g.N * g.outC + row, &tfull[st]);
        }
      }
      }();
      if (tc::aborted(watch))  // the copies of the last stages land before exit
        for (int i = gs > W2_STAGES ? gs - W2_STAGES : 0; i < gs; ++i)
          tc::drain_wait(&tfull[i % W2_STAGES], (i / W2_STAGES) & 1, g.wait_limit);
    }
    __syncwarp();
  } else if (warp == W2_MMA_WARP) {
    // ------------------------------ MMA ------------------------------
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32_amn(W_BM, bn);
      int gs = 0, it = 0;
      [&]() {
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const WTile T = wtile_of(g, t, mtiles, ntn, splits, per, total_chunks, bn);
        if (T.t_begin >= T.t_end) continue;
        const int acc = it & 1;
        if (it >= 2 && !tc::wait(watch, &acc_empty[acc], ((it >> 1) - 1) & 1)) return;
        tc::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * bn);
        for (int tt = T.t_begin; tt < T.t_end; ++tt, ++gs) {
          const int st = gs % W2_STAGES;
          const int s = tt - T.t_begin;
          if (!tc::wait(watch, &full[st], (gs / W2_STAGES) & 1) ||
              !tc::wait(watch, &tfull[st], (gs / W2_STAGES) & 1))
            return;
          tc::tc_fence_after();
          const uint32_t sA = sA0 + st * PARTS * W2_A_STAGE, sB = sB0 + st * PARTS * b_stage;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (SPLIT) {  // lo x hi + hi x lo + hi x hi
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + W2_A_STAGE + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + j * 32), idesc, (s | j) != 0 ? 1u : 0u);
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + b_stage + j * 32), idesc, 1u);
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + j * 32), idesc, 1u);
            } else {
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + j * 32), idesc, (s | j) != 0 ? 1u : 0u);
            }
          }
          tc::umma_commit(&empty[st]);
        }
        tc::umma_commit(&acc_full[acc]);
        ++it;
      }
      }();
      if (tc::aborted(watch)) {  // every UMMA issued so far completes before exit
        tc::umma_commit(drain);
        tc::drain_wait(drain, 0, g.wait_limit);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ------------------------------
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const WTile T = wtile_of(g, t, mtiles, ntn, splits, per, total_chunks, bn);
      if (T.t_begin >= T.t_end) continue;
      const int acc = it & 1;
      if (!tc::wait(watch, &acc_full[acc], (it >> 1) & 1)) break;
      tc::tc_fence_after();
      const int c = T.cm0 + warp * 32 + lane;  // channel within the group
      // element (o, k, c) at o * Cg*kk + k * sk + c * sc (grad_weight, or its
      // tap-major copy)
      const long long ostride = (long long)g.Cg * g.kk;
      float* dst = gw + (long long)(T.gi * g.Og + T.o0) * ostride + (long long)T.k * sk +
                   (long long)c * sc;
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(acc * bn);
      for (int cb = 0; cb < bn; cb += 8) {
        float vv[8];
        tc::tmem_ld8(ta + (uint32_t)cb, vv);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j) red_add_f32(dst + (long long)(cb + j) * ostride, vv[j]);
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
      ++it;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == W2_MMA_WARP) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, (uint32_t)tcols);
  }
}

// ---------------------------------------------------------------------------
// bwd_weight_col: the weight gradient from the column buffer written by the
// grad-column epilogue (col[k][q][C], TF32-rounded; low parts kk*NP rows
// further in 3xTF32):  gW'[c, o] += sum_q col[k][q][c] go[q, o]  (.mm:842-880)
// as a dense tcgen05 GEMM with both operands brought in by TMA.  Tiles as in
// bwd_weight_tc: (tap k, 128 channels, bn out channels, group, pixel range).
//   warps 0-3  epilogue: accumulator -> fp32 reductions into grad_weight, or
//              into a tap-major copy gwt[o][k][c] that the caller transposes
//              into place (a warp's 32 rows of one tap and out channel are
//              then one 128-byte line; in grad_weight's own [o][c][k] order
//              they are kh*kw floats apart)
//   warp  4    MMA issue
//   warp  5    TMA producer: per 32-pixel K step, four 32-channel blocks of
//              col (MN-major operand, 128-byte swizzle with 32-byte atoms)
//              and bn go_r rows
// Rows of a K step past an image's last pixel read the next pixels' columns;
// their go_r columns are zero (padding / out of range), so they add nothing.
// The M side is a 128-row slot of the group's (tap, channel) rows, as in
// bwd_data_tc: 128 channels of one tap, or 128 / Cg taps of 32 or 64
// channels; rows past the last tap are computed and dropped.
// ---------------------------------------------------------------------------
constexpr int WC_THREADS = 192;
constexpr int WC_MMA_WARP = 4, WC_TMA_WARP = 5;

struct WCTile {
  int slot, o0, gi, t_begin, t_end;
};
__device__ __forceinline__ WCTile wctile_of(int t, int nslots, int ntn, int splits, int per,
                                            int total_chunks, int bn) {
  WCTile T;
  const int sp = t % splits;
  int r = t / splits;
  T.o0 = (r % ntn) * bn;
  r /= ntn;
  T.slot = r % nslots;
  T.gi = r / nslots;
  T.t_begin = sp * per;
  T.t_end = min(total_chunks, T.t_begin + per);
  return T;
}

template <bool SPLIT>
__global__ void __launch_bounds__(WC_THREADS, 1)
bwd_weight_col_kernel(Geom g, const __grid_constant__ CUtensorMap colmap,
                      const __grid_constant__ CUtensorMap gomap, int bn, int tcols,
                      float* __restrict__ gw, int sk, int sc, int nslots, int ntn, int splits,
                      int per, int ntiles) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw_u32 & 1023u)) & 1023u);
  constexpr int STAGES = SPLIT ? 2 : 4;
  constexpr int PARTS = SPLIT ? 2 : 1;
  const uint32_t sA0 = tc::smem_u32(smem);
  const uint32_t b_stage = (uint32_t)bn * 128;
  const uint32_t sB0 = sA0 + STAGES * PARTS * W2_A_STAGE;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * PARTS * (W2_A_STAGE + b_stage));
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const tc::Watch watch{abort_flag, &g_tc_bwd_status, kStatusBwdWeight, g.wait_limit};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pchunks = (g.P + 31) >> 5;
  const int total_chunks = g.N * pchunks;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&acc_full[a], 1);
      tc::mbar_init(&acc_empty[a], 4);
    }
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == WC_MMA_WARP) {
    tc::tmem_alloc(tmem_slot, (uint32_t)tcols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == WC_TMA_WARP) {
    if (lane == 0 && !g.no_async) {
      const int lo_rows = g.kk * (int)g.NP;  // row offset of the low parts
      int gs = 0;  // stages filled so far
      [&]() {
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const WCTile T = wctile_of(t, nslots, ntn, splits, per, total_chunks, bn);
        // the four 32-row blocks of the slot: (tap, channel) of each
        int bk[4], bx[4];
#pragma unroll
        for (int mb = 0; mb < 4; ++mb) {
          const int row = T.slot * 128 + mb * 32;
          bk[mb] = row / g.Cg;
          bx[mb] = T.gi * g.Cg + (row - bk[mb] * g.Cg);
        }
        for (int tt = T.t_begin; tt < T.t_end; ++tt, ++gs) {
          const int st = gs % STAGES;
          const int u = gs / STAGES;
          const int n = tt / pchunks;
          const int p0 = (tt - n * pchunks) << 5;
          if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return;
          tc::mbar_arrive_expect_tx(&full[st], PARTS * (W2_A_STAGE + b_stage));
          const uint32_t sA = sA0 + st * PARTS * W2_A_STAGE;
#pragma unroll
          for (int mb = 0; mb < 4; ++mb) {
            // a block past the last tap reads rows beyond the plane (zero fill, or
            // the low plane in 3xTF32); its accumulator rows are dropped
            const int y = bk[mb] * (int)g.NP + n * g.P + p0;
            tc::tma_load_2d(sA + mb * W_LBO, &colmap, bx[mb], y, &full[st]);
            if constexpr (SPLIT)
              tc::tma_load_2d(sA + W2_A_STAGE + mb * W_LBO, &colmap, bx[mb], lo_rows + y,
                              &full[st]);
          }
          const int row = n * g.outC + T.gi * g.Og + T.o0;
          const uint32_t sB = sB0 + st * PARTS * b_stage;
          tc::tma_load_2d(sB, &gomap, p0, row, &full[st]);
          if constexpr (SPLIT)
            tc::tma_load_2d(sB + b_stage, &gomap, p0, g.N * g.outC + row, &full[st]);
        }
      }
      }();
      if (tc::aborted(watch))  // the copies of the last stages land before exit
        for (int i = gs > STAGES ? gs - STAGES : 0; i < gs; ++i)
          tc::drain_wait(&full[i % STAGES], (i / STAGES) & 1, g.wait_limit);
    }
    __syncwarp();
  } else if (warp == WC_MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = idesc_tf32_amn(W_BM, bn);
      int gs = 0, it = 0;
      [&]() {
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const WCTile T = wctile_of(t, nslots, ntn, splits, per, total_chunks, bn);
        if (T.t_begin >= T.t_end) continue;
        const int acc = it & 1;
        if (it >= 2 && !tc::wait(watch, &acc_empty[acc], ((it >> 1) - 1) & 1)) return;
        tc::tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(acc * bn);
        for (int tt = T.t_begin; tt < T.t_end; ++tt, ++gs) {
          const int st = gs % STAGES;
          const int s = tt - T.t_begin;
          if (!tc::wait(watch, &full[st], (gs / STAGES) & 1)) return;
          tc::tc_fence_after();
          const uint32_t sA = sA0 + st * PARTS * W2_A_STAGE, sB = sB0 + st * PARTS * b_stage;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (SPLIT) {  // lo x hi + hi x lo + hi x hi
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + W2_A_STAGE + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + j * 32), idesc, (s | j) != 0 ? 1u : 0u);
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + b_stage + j * 32), idesc, 1u);
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + j * 32), idesc, 1u);
            } else {
              tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                            tc::sdesc_sw128(sB + j * 32), idesc, (s | j) != 0 ? 1u : 0u);
            }
          }
          tc::umma_commit(&empty[st]);
        }
        tc::umma_commit(&acc_full[acc]);
        ++it;
      }
      }();
      if (tc::aborted(watch)) {  // every UMMA issued so far completes before exit
        tc::umma_commit(drain);
        tc::drain_wait(drain, 0, g.wait_limit);
      }
    }
    __syncwarp();
  } else {
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
      const WCTile T = wctile_of(t, nslots, ntn, splits, per, total_chunks, bn);
      if (T.t_begin >= T.t_end) continue;
      const int acc = it & 1;
      if (!tc::wait(watch, &acc_full[acc], (it >> 1) & 1)) break;
      tc::tc_fence_after();
      const int row = T.slot * 128 + warp * 32 + lane;  // (tap, channel) row of the group
      const int k = row / g.Cg, c = row - k * g.Cg;
      const bool live = k < g.kk;
      // element (o, k, c) at o * Cg*kk + k * sk + c * sc
      const long long ostride = (long long)g.Cg * g.kk;
      float* dst = gw + (long long)(T.gi * g.Og + T.o0) * ostride + (long long)k * sk +
                   (long long)c * sc;
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(acc * bn);
      for (int cb = 0; cb < bn; cb += 8) {
        float vv[8];
        tc::tmem_ld8(ta + (uint32_t)cb, vv);
        tc::tmem_ld_wait();
        if (live) {
#pragma unroll
          for (int j = 0; j < 8; ++j) red_add_f32(dst + (long long)(cb + j) * ostride, vv[j]);
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
      ++it;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == WC_MMA_WARP) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, (uint32_t)tcols);
  }
}

// wb_t[(g*kk + k)*Cg + c][o] = tf32(W[g*Og + o][c][k])  (B of bwd_data: rows = channels);
// with `split`, the low parts follow in rows G*kk*Cg ..  Per group a 32 x 32
// tile transpose of W viewed as [o][c*kk + k]: coalesced on both sides.
__device__ __forceinline__ void pack_weight_bwd_tile(int bx, int by, int gi,
                                                     const float* __restrict__ w,
                                                     float* __restrict__ wb, const Geom& g,
                                                     int split) {
  __shared__ float tile[32][33];
  const int CK = g.Cg * g.kk;
  const int o0 = by * 32, ck0 = bx * 32;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const float* src = w + (long long)gi * g.Og * CK;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int o = o0 + ty + i, ck = ck0 + tx;
    if (o < g.Og && ck < CK) tile[ty + i][tx] = __ldg(src + (long long)o * CK + ck);
  }
  __syncthreads();
  const long long lo = (long long)g.G * g.kk * g.Cg * g.Og;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int ck = ck0 + ty + i, o = o0 + tx;
    if (o < g.Og && ck < CK) {
      const int c = ck / g.kk, k = ck - c * g.kk;
      const long long idx = ((long long)(gi * g.kk + k) * g.Cg + c) * g.Og + o;
      const float v = tile[tx][ty + i];
      const float hi = tc::to_tf32(v);
      wb[idx] = hi;
      if (split) wb[lo + idx] = tc::to_tf32(v - hi);
    }
  }
}
__global__ void __launch_bounds__(256) tc_pack_weight_bwd_kernel(const float* __restrict__ w,
                                                                 float* __restrict__ wb, Geom g,
                                                                 int split) {
  pack_weight_bwd_tile(blockIdx.x, blockIdx.y, blockIdx.z, w, wb, g, split);
}

int weight_bn(const Geom& g) { return g.Og <= 256 ? g.Og : 256; }
// 128-row slots of a group's (tap, channel) rows (= kk * Cg / 128 when
// Cg % 128 == 0)
int weight_slots(const Geom& g) { return (g.kk * g.Cg + 127) / 128; }

// Tiles of the weight-gradient kernels and their pixel-range splits: the
// split count minimises the busiest CTA's time, modelled as rounds of tiles x
// (K steps per tile + `tile_cost`, a tile's fixed cost in K steps: pipeline
// fill and the grad_weight reductions), with >= 8 K steps per tile.
struct WSplit {
  int mtiles, ntn, splits, per;
  long long ntiles;
};
WSplit weight_split(const Geom& g, int bn, int num_sms, int tile_cost) {
  WSplit w;
  w.mtiles = g.Cg / W_BM;  // 128-channel tiles per tap (gather kernel)
  w.ntn = g.Og / bn;
  const long long base = (long long)weight_slots(g) * w.ntn * g.G;
  const int pchunks = (g.P + 31) / 32;
  const int total_chunks = g.N * pchunks;
  const long long max_splits = (total_chunks + 7) / 8 > 0 ? (total_chunks + 7) / 8 : 1;
  long long splits = 1, best = -1;
  for (long long sp = 1; sp <= max_splits && sp * base <= 64LL * num_sms; ++sp) {
    const long long rounds = (base * sp + num_sms - 1) / num_sms;
    const long long cost = rounds * ((total_chunks + sp - 1) / sp + tile_cost);
    if (best < 0 || cost < best) {
      best = cost;
      splits = sp;
    }
  }
  w.splits = (int)splits;
  w.per = (int)((total_chunks + splits - 1) / splits);
  w.ntiles = base * splits;
  return w;
}

// ---------------------------------------------------------------------------
// bwd_fused_tc: the whole TF32 tensor-core backward of one (pixel tile,
// slot) in one persistent kernel, for out channels per group <= 256:
//   GEMM1  gcol[q, r] = sum_o go[q, o] W[o, r]                      (.mm:820-821)
//          q = 128 pixels (four 32-pixel blocks, one per tensor-memory lane
//          quarter), r = a 128-row slot of the group's (tap, channel) rows,
//          as in bwd_data_tc;
//   epilogue (16 warps, one per (32-pixel block, 32-channel chunk) of the
//          tile): as epilogue_chunk -- col2im with 16-byte vector reductions
//          (deform_conv2d.metal:141-204), the coordinate / mask gradients
//          from four per-corner sums (deform_conv2d.metal:225-295) -- except
//          that the sampled column values mask * bilinear(x) (TF32) go to a
//          shared-memory column tile, laid out as the MN-major operand of
//   GEMM2  gW[r, o] += sum_q col[q, r] go[q, o]                      (.mm:842-880)
//          A = the column tile, B = go_r rows (K-major), accumulated in
//          tensor memory over all of the CTA's tiles of the slot and reduced
//          into the tap-major grad_weight copy once per slot.
// The columns never leave the SM, and there is no column buffer in HBM.  A
// warp's 4 KB block of the column tile (32 pixel rows x 32 channels in the
// 32-byte-atom swizzle) also serves as its transpose buffer: the grad-column
// rows are written there, read by the gather and the scatter, and then
// overwritten by the column values of the same pixels.
// Work items are (slot, pixel tile) in slot-major order.  When the slots fit
// the grid, every slot gets the same `ranges` contiguous pixel-tile ranges,
// one CTA each (CTA c: slot c % slots, range c / slots), so at any moment the
// CTAs of all slots work on the same few pixel tiles and their inputs,
// grad_out rows and grad-input lines are shared in L2; the weight-gradient
// accumulator is drained once, at the end.  Otherwise (`ranges` 0) the items
// are cut into one contiguous range per CTA, which touches one or two slots.
//   warp 0      TMA producer: per item, the GEMM1 stages of bwd_data_tc and,
//               one item behind, 4 GEMM2 stages (Og rows x 32 pixels of go_r)
//   warp 1      MMA issue: GEMM1 of item i, then GEMM2 of item i - 1
//   warps 2-17  epilogue
// Shared memory: 4 ring stages of 32 KB (both GEMMs), the 64 KB column tile,
// the sampling plans (2 KB a warp), barriers.  Tensor memory: two 128-column
// GEMM1 accumulators and the GEMM2 accumulator (Og <= 256 columns).
// ---------------------------------------------------------------------------
constexpr int F_TMA_WARP = 0, F_MMA_WARP = 1, F_EPI_WARP0 = 2, F_EPI_WARPS = 16;
constexpr int F_THREADS = (F_EPI_WARP0 + F_EPI_WARPS) * 32;  // 576
constexpr int F_STAGES = 4;  // 4 x 32 KB: GEMM2 of an item can have all four go_r blocks in flight
constexpr int F_STAGE = 32768;        // GEMM1: go 16 KB + W 16 KB; GEMM2: go Og x 128 B
constexpr int F_COL = 4 * 16384;      // the column tile
constexpr int F_PLANS = F_EPI_WARPS * 32 * (int)sizeof(PixPlan);
constexpr int F_BAR_BYTES = 256;

size_t fused_smem_bytes() { return (size_t)F_STAGES * F_STAGE + F_COL + F_PLANS + F_BAR_BYTES + 1024; }

struct FItem {
  int gi, sl, mt;
};
__device__ __forceinline__ FItem fitem(long long u, int mtiles, int nslots) {
  FItem it;
  it.mt = (int)(u % mtiles);
  const long long r = u / mtiles;
  it.sl = (int)(r % nslots);
  it.gi = (int)(r / nslots);
  return it;
}

// Image, go_r row and first-pixel coordinate of each 32-pixel block of a
// tile (a block past the last image reads past the row end: zero fill).
__device__ __forceinline__ void fblocks(const Geom& g, const FItem& it, int bpi, int nblocks,
                                        int (&arow)[4], int (&ax)[4]) {
#pragma unroll
  for (int mb = 0; mb < 4; ++mb) {
    const int b = it.mt * 4 + mb;
    const int n = b < nblocks ? b / bpi : 0;
    arow[mb] = n * g.outC + it.gi * g.Og;
    ax[mb] = b < nblocks ? (b - n * bpi) * 32 : bpi * 32;
  }
}

// Byte offset of channels 8 * gran .. 8 * gran + 7 (the 32-byte granule
// `gran`, + 16 for its upper half) of pixel row `px` in a warp's 4 KB block:
// the MN-major, 32-byte-atom swizzled layout of a tcgen05 TF32 operand (K
// row px of 128 bytes, granule position gran ^ (px % 4), rows grouped by 4
// at W_SBO).
__device__ __forceinline__ uint32_t cblk(int px, int gran) {
  return (uint32_t)((px >> 2) * W_SBO + (px & 3) * 128 + (((gran ^ px) & 3) << 5));
}
// ---- storage formats of the fused backward ----
// kF32: fp32 tensors, TF32 operands (kind::tf32); kBF16s / kF16s: bf16 / fp16
// tensors, 16-bit operands (kind::f16) -- the gathers read 16-bit corner
// values, the column tile holds 16-bit values -- with fp32 accumulation in
// tensor memory and fp32 grad-input, offset, mask and weight reductions.
enum : int { kF32 = 0, kBF16s = 1, kF16s = 2 };

// Offset / mask element i as fp32.
template <int FMT>
__device__ __forceinline__ float fld(const void* p, long long i) {
  if constexpr (FMT == kBF16s) {
    return __uint_as_float((uint32_t)__ldg(static_cast<const unsigned short*>(p) + i) << 16);
  } else if constexpr (FMT == kF16s) {
    return __half2float(__ushort_as_half(__ldg(static_cast<const unsigned short*>(p) + i)));
  } else {
    return __ldg(static_cast<const float*>(p) + i);
  }
}
// The two 16-bit values of a 32-bit word (low half first) as fp32, and back
// (round to nearest).
template <int FMT>
__device__ __forceinline__ float h_lo(uint32_t w) {
  if constexpr (FMT == kF16s) return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
  else return __uint_as_float(w << 16);
}
template <int FMT>
__device__ __forceinline__ float h_hi(uint32_t w) {
  if constexpr (FMT == kF16s) return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
  else return __uint_as_float(w & 0xffff0000u);
}
template <int FMT>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  if constexpr (FMT == kF16s) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}
// Byte offset of 16-byte chunk q (channels 8q .. 8q + 7) of pixel row px in
// a warp's 16-bit column block: the MN-major operand of a kind::f16 GEMM with
// the 64-byte swizzle -- K rows of 64 bytes (32 channels), chunk position
// q ^ ((px / 2) % 4), rows grouped by 8 at W_SBO.
__device__ __forceinline__ uint32_t cblk16(int px, int q) {
  return (uint32_t)(px * 64 + (((q ^ (px >> 1)) & 3) << 4));
}
// Shared-memory descriptors of 64-byte-swizzled operands (sm100 version 1):
// MN-major (32-element blocks W_LBO apart, 8-row K groups W_SBO apart) and
// K-major (8-row groups of 64-byte rows, W_SBO apart).
__device__ __forceinline__ uint64_t sdesc_sw64_mn(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(W_LBO >> 4) << 16) |
         ((uint64_t)(W_SBO >> 4) << 32) | (1ull << 46) | (4ull << 61);
}
__device__ __forceinline__ uint64_t sdesc_sw64_k(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | (1ull << 16) | ((uint64_t)(W_SBO >> 4) << 32) |
         (1ull << 46) | (4ull << 61);
}
// 16-byte read-only global load (8 16-bit values).
__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  uint4 r;
  asm("ld.global.nc.v4.b32 {%0, %1, %2, %3}, [%4];"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}

__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
__device__ __forceinline__ float4 ld_shared_f4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

// One epilogue warp, one item: 32 pixel rows (tensor-memory lane quarter) x
// 32 channels of tap k.  As epilogue_chunk, with the warp's column block `tb`
// as the transpose buffer and the column values stored there at the end of
// each group of 8 pixels, once the gather and the scatter of those pixels
// have read their grad-column rows.  16-bit formats: the corner values come
// from the 16-bit NHWC copy (16 bytes a lane and corner), the column values
// are rounded to the tensors' 16-bit type into the first 2 KB of the block
// (K group i of 512 bytes lies over grad-column rows 4i .. 4i + 3, read in
// pass i / 2 <= i).
template <int FMT>
__device__ __forceinline__ void fused_chunk(const Geom& g, const float (&vals)[32], int gch0,
                                            int lane, uint32_t tb, PixPlan* plan,
                                            const void* __restrict__ xt,
                                            float* __restrict__ gxt, float* __restrict__ goff,
                                            float* __restrict__ gmask) {
  const int quad = lane & 3, sub = lane >> 2;
  const int zoff = g.N * g.HW * g.C;
  // Bank spreading: in the swizzled block, rows r and r + 4 (the transpose
  // writes, a lane a row) and rows 8i + 2s, 8i + 2s + 1 (the gather's and
  // the column values' lanes) put the same 16-byte half of a granule on the
  // same banks; lanes with bit 2 set take the two halves in the other order,
  // so every 16-byte access of a quarter warp hits a different bank group.
  const int hs = (lane >> 2) & 1;
  {  // this lane's pixel row into the block, 16 bytes at a time
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int a = 4 * j, b = 4 * (j ^ 1);  // pieces j and j ^ 1 of the row
      tc::st_shared_v4(tb + cblk(lane, j >> 1) + (((j & 1) ^ hs) << 4),
                       hs ? vals[b] : vals[a], hs ? vals[b + 1] : vals[a + 1],
                       hs ? vals[b + 2] : vals[a + 2], hs ? vals[b + 3] : vals[a + 3]);
    }
  }
  __syncwarp();
  // corner loads: channels 8 quad .. 8 quad + 7
  const float* xq = static_cast<const float*>(xt) + gch0 + quad * 8;
  const unsigned short* xq16 = static_cast<const unsigned short*>(xt) + gch0 + quad * 8;
#pragma unroll 2
  for (int i = 0; i < 4; ++i) {
    const int px = i * 8 + sub;
    const PixPlan pl = plan[px];
    const bool live = pl.idx.x >= 0;
    const float m = pl.geo.z;
    const float mw[4] = {m * pl.w.x, m * pl.w.y, m * pl.w.z, m * pl.w.w};
    float d1 = 0.f, d2 = 0.f, d3 = 0.f, d4 = 0.f;
    float cv[8];  // column values (mask * bilinear)
#pragma unroll
    for (int e = 0; e < 8; ++e) cv[e] = 0.f;
    if (live) {
      const float4 l0 = ld_shared_f4(tb + cblk(px, quad) + (hs << 4));
      const float4 l1 = ld_shared_f4(tb + cblk(px, quad) + ((hs ^ 1) << 4));
      const float4 ga = hs ? l1 : l0, gb = hs ? l0 : l1;
      const float gc[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
      float a[8], b[8], c[8], d[8];
      if constexpr (FMT == kF32) {
        ldg_f8(xq + (unsigned)pl.cidx.x, a);  // dropped corners: zero row
        ldg_f8(xq + (unsigned)pl.cidx.y, b);
        ldg_f8(xq + (unsigned)pl.cidx.z, c);
        ldg_f8(xq + (unsigned)pl.cidx.w, d);
      } else {
        const uint4 ua = ldg_u4(xq16 + (unsigned)pl.cidx.x), ub = ldg_u4(xq16 + (unsigned)pl.cidx.y);
        const uint4 uc = ldg_u4(xq16 + (unsigned)pl.cidx.z), ud = ldg_u4(xq16 + (unsigned)pl.cidx.w);
        const uint32_t wa[4] = {ua.x, ua.y, ua.z, ua.w}, wb[4] = {ub.x, ub.y, ub.z, ub.w};
        const uint32_t wc[4] = {uc.x, uc.y, uc.z, uc.w}, wd[4] = {ud.x, ud.y, ud.z, ud.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          a[2 * e] = h_lo<FMT>(wa[e]); a[2 * e + 1] = h_hi<FMT>(wa[e]);
          b[2 * e] = h_lo<FMT>(wb[e]); b[2 * e + 1] = h_hi<FMT>(wb[e]);
          c[2 * e] = h_lo<FMT>(wc[e]); c[2 * e + 1] = h_hi<FMT>(wc[e]);
          d[2 * e] = h_lo<FMT>(wd[e]); d[2 * e + 1] = h_hi<FMT>(wd[e]);
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        d1 = fmaf(gc[e], a[e], d1);
        d2 = fmaf(gc[e], b[e], d2);
        d3 = fmaf(gc[e], c[e], d3);
        d4 = fmaf(gc[e], d[e], d4);
        cv[e] = mw[0] * a[e] + mw[1] * b[e] + mw[2] * c[e] + mw[3] * d[e];
      }
    }
    // the four sums over the pixel's 4 lanes; lanes 0, 1, 2 of the pixel
    // reduce d/dh, d/dw, d/dm into memory
    d1 += __shfl_xor_sync(0xffffffffu, d1, 1);
    d2 += __shfl_xor_sync(0xffffffffu, d2, 1);
    d3 += __shfl_xor_sync(0xffffffffu, d3, 1);
    d4 += __shfl_xor_sync(0xffffffffu, d4, 1);
    d1 += __shfl_xor_sync(0xffffffffu, d1, 2);
    d2 += __shfl_xor_sync(0xffffffffu, d2, 2);
    d3 += __shfl_xor_sync(0xffffffffu, d3, 2);
    d4 += __shfl_xor_sync(0xffffffffu, d4, 2);
    {
      const float dh = m * ((1.f - pl.geo.y) * (d3 - d1) + pl.geo.y * (d4 - d2));
      const float dw = m * ((1.f - pl.geo.x) * (d2 - d1) + pl.geo.x * (d4 - d3));
      const float dm = (pl.w.x * d1 + pl.w.y * d2 + pl.w.z * d3 + pl.w.w * d4) *
                       mask_grad_scale(g, m);
      const float v = quad == 0 ? dh : (quad == 1 ? dw : dm);
      float* dst = quad == 2 ? gmask + (live ? pl.idx.y : 0)
                             : goff + (live ? pl.idx.x : 0) + (quad == 1 ? g.P : 0);
      red_add_f32_if(live && quad < (g.use_mask ? 3 : 2), dst, v);
    }
    // col2im: 8 lanes per pixel, 4 channels each (each quarter warp's 16-byte
    // reductions fill one pixel's 128-byte line); lanes L and L ^ 4 hold the
    // plans of the pixel pair (i * 8 + 2 (sub / 2), + 1) that lanes
    // L & ~7 .. L | 7 reduce
    const int oc[4] = {__shfl_xor_sync(0xffffffffu, pl.cidx.x, 4),
                       __shfl_xor_sync(0xffffffffu, pl.cidx.y, 4),
                       __shfl_xor_sync(0xffffffffu, pl.cidx.z, 4),
                       __shfl_xor_sync(0xffffffffu, pl.cidx.w, 4)};
    const float omw[4] = {__shfl_xor_sync(0xffffffffu, mw[0], 4),
                          __shfl_xor_sync(0xffffffffu, mw[1], 4),
                          __shfl_xor_sync(0xffffffffu, mw[2], 4),
                          __shfl_xor_sync(0xffffffffu, mw[3], 4)};
    const bool olive = __shfl_xor_sync(0xffffffffu, (int)live, 4) != 0;
    const int j = lane & 7;
    float* gq = gxt + gch0 + j * 4;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const bool own = h == (sub & 1);
      const bool hl = own ? live : olive;
      const int rp = i * 8 + (sub & ~1) + h;
      const float4 g4 = ld_shared_f4(tb + cblk(rp, j >> 1) + ((j & 1) << 4));
      const int cis[4] = {own ? pl.cidx.x : oc[0], own ? pl.cidx.y : oc[1],
                          own ? pl.cidx.z : oc[2], own ? pl.cidx.w : oc[3]};
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        // dropped corners (the zero row) and void samples are not reduced
        const bool on = hl && cis[cc] != zoff;
        const float wc = own ? mw[cc] : omw[cc];
        red_add_v4_if(on, gq + (unsigned)(on ? cis[cc] : 0), wc * g4.x, wc * g4.y, wc * g4.z,
                      wc * g4.w);
      }
    }
    // the grad-column rows of these 8 pixels are read: their column values
    // take their place (TF32-rounded; 0 for void samples and past the image)
    __syncwarp();
    if constexpr (FMT == kF32) {
      float hv[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) hv[e] = tc::to_tf32(hs ? cv[e ^ 4] : cv[e]);
      tc::st_shared_v4(tb + cblk(px, quad) + (hs << 4), hv[0], hv[1], hv[2], hv[3]);
      tc::st_shared_v4(tb + cblk(px, quad) + ((hs ^ 1) << 4), hv[4], hv[5], hv[6], hv[7]);
    } else {
      st_shared_u4(tb + cblk16(px, quad), pack2<FMT>(cv[0], cv[1]), pack2<FMT>(cv[2], cv[3]),
                   pack2<FMT>(cv[4], cv[5]), pack2<FMT>(cv[6], cv[7]));
    }
  }
}

// FMT kF32: TF32 operands, K steps of 32 out channels (GEMM1) and 8 pixels
// (GEMM2, 4 UMMAs a 32-pixel block), 128-byte swizzles.  kBF16s / kF16s:
// 16-bit operands (kind::f16), K steps of 64 out channels and 16 pixels (2
// UMMAs a block); go_r blocks and GEMM2's B in the 64-byte swizzle (32 pixels
// x 2 bytes a row), the same stage bytes and descriptor strides.
template <int FMT>
__global__ void __launch_bounds__(F_THREADS, 1)
bwd_fused_tc_kernel(Geom g, const __grid_constant__ CUtensorMap amap,
                    const __grid_constant__ CUtensorMap bmap,
                    const __grid_constant__ CUtensorMap g2map, int bpi, int nblocks, int mtiles,
                    int nslots, long long nitems, int ranges, const void* __restrict__ xt,
                    const void* __restrict__ off, const void* __restrict__ mask,
                    float* __restrict__ gxt, float* __restrict__ goff,
                    float* __restrict__ gmask, float* __restrict__ gwt) {
  constexpr bool H16 = FMT != kF32;
  constexpr int KO = H16 ? 64 : 32;  // out channels of a GEMM1 K step
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw_u32 & 1023u)) & 1023u);
  const uint32_t ring = tc::smem_u32(smem);
  const uint32_t colt = ring + F_STAGES * F_STAGE;
  PixPlan* plans = reinterpret_cast<PixPlan*>(smem + F_STAGES * F_STAGE + F_COL);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + F_STAGES * F_STAGE + F_COL + F_PLANS);
  uint64_t* empty = full + F_STAGES;
  uint64_t* acc_full = empty + F_STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* col_full = acc_empty + 2;   // per 32-pixel K block: its 4 epilogue warps wrote it
  uint64_t* col_empty = col_full + 4;   // per K block: GEMM2 has read it
  uint64_t* acc2_full = col_empty + 4;
  uint64_t* acc2_empty = acc2_full + 1;
  uint64_t* drain = acc2_empty + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const tc::Watch watch{abort_flag, &g_tc_bwd_status, kStatusBwdData | kStatusBwdWeight,
                        g.wait_limit};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // 32-out-channel K steps of GEMM1; a partial last one reads zero weights
  // past Og (the weight map ends there), so the go_r rows it loads add nothing
  const int ochunks = (g.Og + KO - 1) / KO;
  // this CTA's items [u0, u0 + n) in slot-major order
  long long u0;
  int n;
  if (ranges > 0) {  // one pixel-tile range of one slot
    const int slots = (int)(nitems / mtiles);
    const int s = (int)blockIdx.x % slots, rg = (int)blockIdx.x / slots;
    const int mt0 = (int)((long long)rg * mtiles / ranges);
    u0 = (long long)s * mtiles + mt0;
    n = (int)((long long)(rg + 1) * mtiles / ranges) - mt0;
  } else {
    u0 = (long long)blockIdx.x * nitems / gridDim.x;
    n = (int)((long long)(blockIdx.x + 1) * nitems / gridDim.x - u0);
  }
  auto seg_of = [&](int i) { return (u0 + i) / mtiles; };  // (group, slot) of item i

  if (tid == 0) {
    for (int s = 0; s < F_STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&acc_full[a], 1);
      tc::mbar_init(&acc_empty[a], F_EPI_WARPS);
    }
    for (int q = 0; q < 4; ++q) {
      tc::mbar_init(&col_full[q], 4);
      tc::mbar_init(&col_empty[q], 1);
    }
    tc::mbar_init(acc2_full, 1);
    tc::mbar_init(acc2_empty, F_EPI_WARPS);
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == F_MMA_WARP) {
    tc::tmem_alloc(tmem_slot, 512);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == F_TMA_WARP) {
    if (lane == 0 && !g.no_async) {
      int gs = 0;  // stages filled so far
      [&]() {
        auto acquire = [&]() -> int {  // next ring stage, once the GEMMs have read it
          const int st = gs % F_STAGES, u = gs / F_STAGES;
          if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return -1;
          return st;
        };
        int arow[4], ax[4];
        for (int i = 0; i <= n; ++i) {
          if (i < n) {  // GEMM1 of item i: go_r blocks (MN-major) and W slot rows
            const FItem it = fitem(u0 + i, mtiles, nslots);
            fblocks(g, it, bpi, nblocks, arow, ax);
            const int brow = it.gi * g.kk * g.Cg + it.sl * 128;
            for (int s = 0; s < ochunks; ++s, ++gs) {
              const int st = acquire();
              if (st < 0) return;
              const uint32_t sA = ring + st * F_STAGE;
              tc::mbar_arrive_expect_tx(&full[st], F_STAGE);
#pragma unroll
              for (int mb = 0; mb < 4; ++mb)
                tc::tma_load_2d(sA + mb * W_LBO, &amap, ax[mb], arow[mb] + s * KO, &full[st]);
              tc::tma_load_2d(sA + 16384, &bmap, s * KO, brow, &full[st]);
            }
          }
          if (i >= 1) {  // GEMM2 of item i - 1: go_r rows of each 32-pixel block
            const FItem it = fitem(u0 + i - 1, mtiles, nslots);
            fblocks(g, it, bpi, nblocks, arow, ax);
            for (int pq = 0; pq < 4; ++pq, ++gs) {
              const int st = acquire();
              if (st < 0) return;
              tc::mbar_arrive_expect_tx(&full[st], (uint32_t)g.Og * (H16 ? 64 : 128));
              tc::tma_load_2d(ring + st * F_STAGE, &g2map, ax[pq], arow[pq], &full[st]);
            }
          }
        }
      }();
      if (tc::aborted(watch))  // the copies of the last stages land before exit
        for (int i = gs > F_STAGES ? gs - F_STAGES : 0; i < gs; ++i)
          tc::drain_wait(&full[i % F_STAGES], (i / F_STAGES) & 1, g.wait_limit);
    }
    __syncwarp();
  } else if (warp == F_MMA_WARP) {
    if (lane == 0) {
      // GEMM1: A = go_r pixels (MN-major), B = W slot rows (K-major);
      // GEMM2: A = column tile (MN-major: channels contiguous), B = go_r rows (K-major)
      const uint32_t amn = 1u << 15;
      const uint32_t idesc1 = FMT == kF16s    ? tc::idesc_f16(128, 128) | amn
                              : FMT == kBF16s ? tc::idesc_bf16(128, 128) | amn
                                              : idesc_tf32_amn(128, 128);
      const uint32_t idesc2 = FMT == kF16s    ? tc::idesc_f16(128, g.Og) | amn
                              : FMT == kBF16s ? tc::idesc_bf16(128, g.Og) | amn
                                              : idesc_tf32_amn(128, g.Og);
      int gs = 0, segs = 0;
      [&]() {
        for (int i = 0; i <= n; ++i) {
          if (i < n) {
            const int acc = i & 1;
            if (i >= 2 && !tc::wait(watch, &acc_empty[acc], ((i >> 1) - 1) & 1)) return;
            tc::tc_fence_after();
            const uint32_t d = tmem + (uint32_t)(acc * 128);
            for (int s = 0; s < ochunks; ++s, ++gs) {
              const int st = gs % F_STAGES;
              if (!tc::wait(watch, &full[st], (gs / F_STAGES) & 1)) return;
              tc::tc_fence_after();
              const uint32_t sA = ring + st * F_STAGE, sB = sA + 16384;
#pragma unroll
              for (int j = 0; j < 4; ++j) {  // 8 (TF32) or 16 (16-bit) out channels each
                if constexpr (H16)
                  tc::umma_bf16(d, sdesc_sw64_mn(sA + j * 2 * W_SBO), tc::sdesc_sw128(sB + j * 32),
                                idesc1, (s | j) != 0 ? 1u : 0u);
                else
                  tc::umma_tf32(d, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                                tc::sdesc_sw128(sB + j * 32), idesc1, (s | j) != 0 ? 1u : 0u);
              }
              tc::umma_commit(&empty[st]);
            }
            tc::umma_commit(&acc_full[acc]);
          }
          if (i >= 1) {
            const int p = i - 1;
            const bool first = p == 0 || seg_of(p) != seg_of(p - 1);
            const bool last = p == n - 1 || seg_of(p + 1) != seg_of(p);
            // the previous slot's accumulator has been drained
            if (first && segs > 0 && !tc::wait(watch, acc2_empty, (segs - 1) & 1)) return;
            tc::tc_fence_after();
            const uint32_t d2 = tmem + 256u;
            for (int pq = 0; pq < 4; ++pq, ++gs) {
              const int st = gs % F_STAGES;
              if (!tc::wait(watch, &col_full[pq], p & 1) ||
                  !tc::wait(watch, &full[st], (gs / F_STAGES) & 1))
                return;
              tc::tc_fence_after();
              const uint32_t sB = ring + st * F_STAGE, sA = colt + pq * 16384;
#pragma unroll
              for (int j = 0; j < (H16 ? 2 : 4); ++j) {  // 8 (TF32) or 16 (16-bit) pixels each
                if constexpr (H16)
                  tc::umma_bf16(d2, sdesc_sw64_mn(sA + j * 2 * W_SBO), sdesc_sw64_k(sB + j * 32),
                                idesc2, (first && pq == 0 && j == 0) ? 0u : 1u);
                else
                  tc::umma_tf32(d2, sdesc_sw128b32_mn(sA + j * 2 * W_SBO),
                                tc::sdesc_sw128(sB + j * 32), idesc2,
                                (first && pq == 0 && j == 0) ? 0u : 1u);
              }
              tc::umma_commit(&empty[st]);
              tc::umma_commit(&col_empty[pq]);
            }
            if (last) {
              tc::umma_commit(acc2_full);
              ++segs;
            }
          }
        }
      }();
      if (tc::aborted(watch)) {  // every UMMA issued so far completes before exit
        tc::umma_commit(drain);
        tc::drain_wait(drain, 0, g.wait_limit);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ------------------------------
    const int e = warp - F_EPI_WARP0;
    const int lq = warp & 3;     // tensor-memory lane quarter: 32-pixel block of the tile
    const int chunk = e >> 2;    // 32-channel chunk of the slot
    PixPlan* plan = plans + e * 32;
    const uint32_t tb = colt + lq * 16384 + chunk * W_LBO;  // this warp's 4 KB block
    const int zoff = g.N * g.HW * g.C;
    int segs = 0;
    [&]() {
      for (int i = 0; i < n; ++i) {
        const FItem it = fitem(u0 + i, mtiles, nslots);
        const int acc = i & 1;
        const int b = it.mt * 4 + lq;
        const int bimg = b < nblocks ? b / bpi : 0;
        const long long qbase = b < nblocks ? (long long)bimg * g.P + (long long)(b - bimg * bpi) * 32 : 0;
        const long long qend = b < nblocks ? (long long)bimg * g.P + g.P : 0;
        const long long row_q = qbase + lane;
        const int row = it.sl * 128 + chunk * 32;  // (tap, channel) row within the group
        const int k = row / g.Cg;
        const bool rows_ok = k < g.kk;
        const int gch0 = it.gi * g.Cg + (row - k * g.Cg);
        const int dgi = gch0 / g.cpg;
        if (!tc::wait(watch, &acc_full[acc], (i >> 1) & 1)) return;
        tc::tc_fence_after();
        float vals[32];
        {
          const uint32_t ta = tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)(acc * 128 + chunk * 32);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float tv[8];
            tc::tmem_ld8(ta + 8 * j, tv);
#pragma unroll
            for (int q = 0; q < 8; ++q) vals[8 * j + q] = tv[q];
          }
          tc::tmem_ld_wait();
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);  // the accumulator is free for item i + 2
        {  // sampling plan of this lane's pixel for (tap k, deformable group dgi)
          PixPlan pl;
          pl.cidx = make_int4(zoff, zoff, zoff, zoff);
          pl.w = make_float4(0.f, 0.f, 0.f, 0.f);
          pl.geo = make_float4(0.f, 0.f, 0.f, 0.f);
          pl.idx = make_int4(-1, 0, 0, 0);
          if (rows_ok && row_q < qend) {
            const int ni = (int)(row_q / g.P);
            const int p = (int)(row_q - (long long)ni * g.P);
            const int oy = p / g.Wo, ox = p - oy * g.Wo;
            const int ki = k / g.kw, kj = k - ki * g.kw;
            const long long oi = off_h_index(g, ni, dgi, k, p);
            float h, w;
            sample_pos(g, oy, ox, ki, kj, fld<FMT>(off, oi), fld<FMT>(off, oi + g.P), h, w);
            const Sample sp = make_sample(h, w, g.H, g.W);
            if (sp.valid) {
              const int nb = ni * g.HW;
              pl.cidx.x = (sp.live & 1u) ? (nb + sp.i1) * g.C : zoff;
              pl.cidx.y = (sp.live & 2u) ? (nb + sp.i2) * g.C : zoff;
              pl.cidx.z = (sp.live & 4u) ? (nb + sp.i3) * g.C : zoff;
              pl.cidx.w = (sp.live & 8u) ? (nb + sp.i4) * g.C : zoff;
              pl.w = make_float4(sp.w1, sp.w2, sp.w3, sp.w4);
              const long long mi = mask_index(g, ni, dgi, k, p);
              float m = 1.f;
              if (g.use_mask) {
                const float raw = fld<FMT>(mask, mi);
                m = g.mask_logits ? 1.f / (1.f + expf(-raw)) : raw;
              }
              pl.geo = make_float4(sp.lh, sp.lw, m, 0.f);
              pl.idx = make_int4((int)oi, (int)mi, 0, 0);
            }
          }
          plan[lane] = pl;
        }
        // GEMM2 of the previous item has read this block of the column tile
        if (i >= 1 && !tc::wait(watch, &col_empty[lq], (i - 1) & 1)) return;
        if (rows_ok) {
          fused_chunk<FMT>(g, vals, gch0, lane, tb, plan, xt, gxt, goff, gmask);
        } else {  // rows past the group's last tap: zero columns
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::st_shared_v4(tb + cblk(lane, j >> 1) + ((j & 1) << 4), 0.f, 0.f, 0.f, 0.f);
        }
        // the column block is complete: visible to the tensor core
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&col_full[lq]);
        if (i == n - 1 || seg_of(i + 1) != seg_of(i)) {
          // the slot's weight gradient: tensor-memory lanes are its rows,
          // columns its out channels; this warp drains 64 of them into the
          // tap-major copy [o][k][c] (a warp's 32 rows: one 128-byte line)
          if (!tc::wait(watch, acc2_full, segs & 1)) return;
          tc::tc_fence_after();
          const int r = it.sl * 128 + lq * 32 + lane;
          const int kr = r / g.Cg, cr = r - kr * g.Cg;
          float* dst = gwt + (long long)(it.gi * g.Og) * g.kk * g.Cg + (long long)kr * g.Cg + cr;
          const long long ostride = (long long)g.kk * g.Cg;
          const uint32_t t2 = tmem + ((uint32_t)(lq * 32) << 16) + 256u;
          for (int cb = chunk * 64; cb < chunk * 64 + 64 && cb < g.Og; cb += 8) {
            float vv[8];
            tc::tmem_ld8(t2 + (uint32_t)cb, vv);
            tc::tmem_ld_wait();
            if (kr < g.kk) {
#pragma unroll
              for (int x = 0; x < 8; ++x) red_add_f32(dst + (long long)(cb + x) * ostride, vv[x]);
            }
          }
          tc::tc_fence_before();
          __syncwarp();
          if (lane == 0) tc::mbar_arrive(acc2_empty);
          ++segs;
        }
      }
    }();
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == F_MMA_WARP) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

}  // namespace

cudaError_t read_bwd_status(int* status, bool clear, cudaStream_t stream) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_tc_bwd_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_tc_bwd_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  *status = v;
  return e;
}

bool tc_bwd_supported(const Geom& g) {
  // channels per group: any multiple of 32 (a 128-row slot of the group's
  // (tap, channel) rows is four 32-channel chunks, each inside one tap)
  return g.Cg % 32 == 0 && g.cpg % 32 == 0 && g.C % 4 == 0 && g.Og % 16 == 0 &&
         (g.Og <= 256 || g.Og % 256 == 0) &&
         g.NP > 0 && (long long)g.N * g.HW * g.C + g.C < (1LL << 31) &&
         (long long)g.N * 2 * g.dg * g.kk * g.P < (1LL << 31);
}

bool tc_wgather_supported(const Geom& g) { return tc_bwd_supported(g) && g.Cg % W_BM == 0; }

cudaError_t launch_tc_prep_go(const Geom& g, const float* go, float* go_r, float* gb,
                              bool split, cudaStream_t stream) {
  if ((long long)g.N * g.outC * g.P == 0) return cudaSuccess;
  const int Ppad = (g.P + 3) & ~3;
  const int pspans = (Ppad + PG_SPAN - 1) / PG_SPAN;
  const long long blocks = (long long)g.N * g.outC * pspans;
  if (blocks > (1LL << 31) - 1) return cudaErrorInvalidValue;
  const int vec = g.P % 4 == 0 && (reinterpret_cast<uintptr_t>(go) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(go_r) & 15u) == 0;
  prep_go_kernel<<<(unsigned)blocks, 256, 0, stream>>>(go, go_r, gb, g.N, g.outC, g.P, Ppad,
                                                       pspans, split ? 1 : 0, vec);
  return cudaGetLastError();
}

cudaError_t launch_tc_pack_weight_bwd(const float* w, float* wbt, const Geom& g, bool split,
                                      cudaStream_t stream) {
  const long long total = (long long)g.G * g.kk * g.Cg * g.Og;
  if (total == 0) return cudaSuccess;
  if ((g.Og + 31) / 32 > 65535 || g.G > 65535) return cudaErrorInvalidValue;
  dim3 grid((g.Cg * g.kk + 31) / 32, (g.Og + 31) / 32, g.G);
  tc_pack_weight_bwd_kernel<<<grid, 256, 0, stream>>>(w, wbt, g, split ? 1 : 0);
  return cudaGetLastError();
}

namespace {
// The fused backward's helpers in one launch (staged input, TF32), as work
// items: [0, nb_prep) prepare a PG_SPAN of a grad_out row each (grad_bias as
// per-item partial sums), the next nb_pack pack a 32 x 32 weight tile each,
// the rest zero 16 KB of an accumulator each (zc[l] items for array l; the
// first item of an array also takes its scalar tail).  A block takes items
// blockIdx.x, + gridDim.x, ...: every block gets a mix of the three kinds.
constexpr int ZERO_ITEM = 4096;  // floats an item zeroes (256 threads x 4 float4)
struct ZeroItems {
  float* zp[4];
  long long zn[4];   // floats of array l
  long long zv[4];   // float4 vectors zeroed as vectors (0: misaligned, all scalar)
  int zitems[4];     // items of array l
  int zcount;
  int total;         // items of all arrays
};
// Zero item b of `z` (256 threads).
__device__ __forceinline__ void zero_item(const ZeroItems& z, int b) {
  int l = 0;
  while (l < z.zcount - 1 && b >= z.zitems[l]) b -= z.zitems[l++];
  float* p = z.zp[l];
  const long long n = z.zn[l], nv = z.zv[l];
  if (nv > 0) {
    float4* p4 = reinterpret_cast<float4*>(p);
    const long long v0 = (long long)b * (ZERO_ITEM / 4);
#pragma unroll
    for (int u = 0; u < ZERO_ITEM / 1024; ++u) {
      const long long v = v0 + u * 256 + threadIdx.x;
      if (v < nv) p4[v] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (b == 0)
      for (long long i = (nv << 2) + threadIdx.x; i < n; i += 256) p[i] = 0.f;
  } else {
    const long long e0 = (long long)b * ZERO_ITEM;
    for (long long i = e0 + threadIdx.x; i < e0 + ZERO_ITEM && i < n; i += 256) p[i] = 0.f;
  }
}
// The items of a ZeroList (host).
bool zero_items(const ZeroList& zl, ZeroItems& z) {
  z = ZeroItems{};
  z.zcount = zl.count;
  long long total = 0;
  for (int l = 0; l < zl.count; ++l) {
    z.zp[l] = zl.ptr[l];
    z.zn[l] = zl.n[l];
    z.zv[l] = (reinterpret_cast<uintptr_t>(zl.ptr[l]) & 15u) == 0 ? zl.n[l] >> 2 : 0;
    const long long items = (zl.n[l] + ZERO_ITEM - 1) / ZERO_ITEM;
    if (items > (1LL << 30)) return false;
    z.zitems[l] = (int)items;
    total += items;
  }
  if (total > (1LL << 30)) return false;
  z.total = (int)total;
  return true;
}
struct Prologue {
  const float* go;
  float* go_r;
  float* gpart;
  const float* w;
  float* wbt;
  ZeroItems z;
  int Ppad, pspans, vec;
  int nb_prep, pack_x, pack_y, nb_pack, total;
};
__global__ void __launch_bounds__(256) bwd_prologue_kernel(Prologue a, Geom g) {
  for (int it = blockIdx.x; it < a.total; it += gridDim.x) {
    int b = it;
    if (b < a.nb_prep) {
      prep_go_block(b, a.go, a.go_r, nullptr, a.gpart, g.N, g.outC, g.P, a.Ppad, a.pspans, 0,
                    a.vec);
    } else if ((b -= a.nb_prep) < a.nb_pack) {
      const int per_g = a.pack_x * a.pack_y;
      const int gi = b / per_g, r = b - gi * per_g;
      pack_weight_bwd_tile(r % a.pack_x, r / a.pack_x, gi, a.w, a.wbt, g, 0);
    } else {
      zero_item(a.z, b - a.nb_pack);
    }
    __syncthreads();  // the shared staging of one item is free before the next
  }
}
}  // namespace

size_t tc_bias_part_floats(const Geom& g) {
  const int Ppad = (g.P + 3) & ~3;
  return (size_t)g.N * g.outC * ((Ppad + PG_SPAN - 1) / PG_SPAN);
}

cudaError_t launch_bwd_prologue(const Geom& g, const float* go, float* go_r, float* gpart,
                                const float* w, float* wbt, const ZeroList& z,
                                cudaStream_t stream) {
  if (g.P == 0 || z.count > 4) return cudaErrorInvalidValue;
  Prologue a{};
  a.go = go;
  a.go_r = go_r;
  a.gpart = gpart;
  a.w = w;
  a.wbt = wbt;
  if (!zero_items(z, a.z)) return cudaErrorInvalidValue;
  const long long zitems = a.z.total;
  a.Ppad = (g.P + 3) & ~3;
  a.pspans = (a.Ppad + PG_SPAN - 1) / PG_SPAN;
  a.vec = g.P % 4 == 0 && (reinterpret_cast<uintptr_t>(go) & 15u) == 0 &&
          (reinterpret_cast<uintptr_t>(go_r) & 15u) == 0;
  const long long prep = (long long)g.N * g.outC * a.pspans;
  a.pack_x = (g.Cg * g.kk + 31) / 32;
  a.pack_y = (g.Og + 31) / 32;
  const long long pack = (long long)a.pack_x * a.pack_y * g.G;
  const long long total = prep + pack + zitems;
  if (total > (1LL << 31) - 1) return cudaErrorInvalidValue;
  a.nb_prep = (int)prep;
  a.nb_pack = (int)pack;
  a.total = (int)total;
  const long long grid = std::min<long long>(total, (long long)device_sm_count() * 8);
  bwd_prologue_kernel<<<(unsigned)grid, 256, 0, stream>>>(a, g);
  return cudaGetLastError();
}

cudaError_t launch_bwd_data_tc(const Geom& g, const float* go_r, bool split, const float* wbt,
                               const float* xt, const float* off, const float* mask, float* gxt,
                               float* goff, float* gmask, float* col, cudaStream_t stream) {
  const int Ppad = (g.P + 3) & ~3;
  CUtensorMap amap, bmap;
  // go_r viewed as N*outC (x2 in 3xTF32) rows of P pixels, Ppad apart: boxes
  // of 32 pixels x 32 rows, MN-major swizzle
  cudaError_t e = make_tmap_2d_f32(&amap, go_r, (uint64_t)g.P,
                                   (uint64_t)g.N * g.outC * (split ? 2 : 1), (uint64_t)Ppad, 32u,
                                   /*atom32=*/true);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d_f32(&bmap, wbt, (uint64_t)g.Og, (uint64_t)g.G * g.kk * g.Cg * (split ? 2 : 1),
                       (uint64_t)g.Og, (uint32_t)D_BN);
  if (e != cudaSuccess) return e;
  const size_t smem = data_smem_bytes(split);
  auto kern = split ? bwd_data_tc_kernel<true> : bwd_data_tc_kernel<false>;
  const int threads = split ? DCfg<true>::THREADS : DCfg<false>::THREADS;
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem);
  if (e != cudaSuccess) return e;
  const int sms = device_sm_count();
  const int bpi = (g.P + 31) / 32;  // 32-pixel blocks per image
  if ((long long)g.N * bpi > (1LL << 30)) return cudaErrorInvalidValue;
  const int nblocks = g.N * bpi;
  const int mtiles = (nblocks + 3) / 4;
  const int nslots = (g.kk * g.Cg + D_BN - 1) / D_BN;
  const long long base = (long long)mtiles * g.G;
  // split the slots so the busiest CTA carries the fewest
  int ksplits = 1;
  long long best = -1;
  for (int ks = 1; ks <= nslots; ++ks) {
    const long long rounds = (base * ks + sms - 1) / sms;
    const long long cost = rounds * ((nslots + ks - 1) / ks);
    if (best < 0 || cost < best) {
      best = cost;
      ksplits = ks;
    }
  }
  const long long ntiles = base * ksplits;
  if (ntiles > (1LL << 30)) return cudaErrorInvalidValue;
  const int grid = (int)(ntiles < sms ? ntiles : sms);
  kern<<<grid, threads, smem, stream>>>(g, amap, bmap, bpi, nblocks, mtiles, nslots, ksplits,
                                         (int)ntiles,
                                         xt, off, mask, gxt, goff, gmask, col);
  return cudaGetLastError();
}

cudaError_t launch_tc_plans(const Geom& g, const float* off, const float* mask, void* plans,
                            cudaStream_t stream) {
  const long long total = (long long)g.N * g.dg * g.kk * g.P;
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  plan_kernel<<<(int)blocks, 256, 0, stream>>>(g, off, mask, static_cast<int4*>(plans));
  return cudaGetLastError();
}

cudaError_t launch_bwd_weight_tc(const Geom& g, const float* go_r, const float* xt,
                                 const void* plans, float* gw, bool tap_major, bool split,
                                 int num_sms, cudaStream_t stream) {
  if (!tc_wgather_supported(g)) return cudaErrorInvalidValue;
  const int bn = weight_bn(g);
  const int Ppad = (g.P + 3) & ~3;
  CUtensorMap gomap;
  cudaError_t e = make_tmap_2d_f32(&gomap, go_r, (uint64_t)Ppad,
                                   (uint64_t)g.N * g.outC * (split ? 2 : 1), (uint64_t)Ppad,
                                   (uint32_t)bn);
  if (e != cudaSuccess) return e;
  const size_t smem = weight_smem_bytes(bn, split);
  auto kern = split ? bwd_weight_tc_kernel<true> : bwd_weight_tc_kernel<false>;
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem);
  if (e != cudaSuccess) return e;
  // a gathered K step costs far more than the tile's fixed work
  const WSplit w = weight_split(g, bn, num_sms, 0);
  if (w.ntiles > (1LL << 30)) return cudaErrorInvalidValue;
  const int grid = (int)(w.ntiles < num_sms ? w.ntiles : num_sms);
  kern<<<grid, W2_THREADS, smem, stream>>>(g, gomap, bn, pow2_cols(2 * bn), xt,
                                            static_cast<const int4*>(plans), gw,
                                            tap_major ? g.Cg : 1, tap_major ? 1 : g.kk, w.mtiles,
                                            w.ntn, w.splits, w.per, (int)w.ntiles);
  return cudaGetLastError();
}

// gwt[o][k][c] -> gw[o][c][k]: one thread per (o, c); a warp reads 32
// consecutive channels of each tap (coalesced) and writes 32 x kk consecutive
// floats.
// With `gpart`: also grad_bias[o] = the sum of the prologue's partial sums
// of out channel o, in a fixed order.
// Block `bb` of `nb` blocks of 256 threads: its share of the (o, c) rows of
// the layout change and of the grad_bias sums.
__device__ __forceinline__ void weight_from_tap_major_blocks(
    long long bb, long long nb, const float* __restrict__ gwt, float* __restrict__ gw, int Cg,
    int kk, long long total, const float* __restrict__ gpart, float* __restrict__ gb, int N,
    int outC, int pspans) {
  const long long stride = nb * 256;
  for (long long i = bb * 256 + threadIdx.x; i < total; i += stride) {
    const long long o = i / Cg;
    const int c = (int)(i - o * Cg);
    const float* src = gwt + o * Cg * kk + c;
    float* dst = gw + i * kk;
    for (int k = 0; k < kk; ++k) dst[k] = __ldg(src + (long long)k * Cg);
  }
  if (gpart == nullptr) return;
  for (long long o = bb * 256 + threadIdx.x; o < outC; o += stride) {
    float t = 0.f;
    for (int n = 0; n < N; ++n) {
      const float* q = gpart + ((long long)n * outC + o) * pspans;
      for (int sp = 0; sp < pspans; ++sp) t += __ldg(q + sp);
    }
    gb[o] = t;
  }
}
__global__ void __launch_bounds__(256) weight_from_tap_major_kernel(
    const float* __restrict__ gwt, float* __restrict__ gw, int Cg, int kk, long long total,
    const float* __restrict__ gpart, float* __restrict__ gb, int N, int outC, int pspans) {
  weight_from_tap_major_blocks(blockIdx.x, gridDim.x, gwt, gw, Cg, kk, total, gpart, gb, N,
                               outC, pspans);
}

// The fused backward's last two jobs in one launch on the caller's stream:
// blocks [0, tiles) transpose the NHWC grad-input accumulator gxt into
// grad_input (NCHW, 64 x 64 tiles), the blocks after them lay out
// grad_weight from its tap-major copy and sum grad_bias
// (weight_from_tap_major_kernel's work).  One launch instead of a transpose
// beside a side-stream layout kernel saves the fork, the join and a launch.
__global__ void __launch_bounds__(256) bwd_finish_kernel(
    const float* __restrict__ gxt, float* __restrict__ gx, int C, int HW, int tiles_x,
    int per_img, int tiles, const float* __restrict__ gwt, float* __restrict__ gw, int Cg,
    int kk, long long total, const float* __restrict__ gpart, float* __restrict__ gb, int N,
    int outC, int pspans) {
  __shared__ float tile[64][65];
  const int b = blockIdx.x;
  if (b < tiles) {
    const int n = b / per_img, r = b - n * per_img;
    transpose4_tile(gxt, gx, HW, C, n, r % tiles_x, r / tiles_x, tile, nullptr);
  } else {
    weight_from_tap_major_blocks(b - tiles, (long long)gridDim.x - tiles, gwt, gw, Cg, kk, total,
                                 gpart, gb, N, outC, pspans);
  }
}

cudaError_t launch_weight_from_tap_major(const float* gwt, float* gw, const Geom& g,
                                         cudaStream_t stream, const float* gpart, float* gb) {
  const long long total = (long long)g.outC * g.Cg;
  if (total == 0 || g.kk == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  const int Ppad = (g.P + 3) & ~3;
  const int pspans = (Ppad + PG_SPAN - 1) / PG_SPAN;
  weight_from_tap_major_kernel<<<(int)blocks, 256, 0, stream>>>(
      gwt, gw, g.Cg, g.kk, total, gb != nullptr ? gpart : nullptr, gb, g.N, g.outC, pspans);
  return cudaGetLastError();
}

bool bwd_finish_fits(const float* gxt, const float* gx, const Geom& g) {
  return transpose4_fits(gxt, gx, g.HW, g.C) &&
         transpose4_tiles(g.N, g.HW, g.C) + 148LL * 16 <= (1LL << 31) - 1;
}

cudaError_t launch_bwd_finish(const float* gxt, float* gx, const float* gwt, float* gw,
                              const Geom& g, const float* gpart, float* gb, cudaStream_t stream) {
  if (!bwd_finish_fits(gxt, gx, g)) return cudaErrorInvalidValue;
  // gxt (N, HW, C) -> grad_input (N, C, HW): rows HW, columns C
  const long long tiles = transpose4_tiles(g.N, g.HW, g.C);
  const long long total = g.kk > 0 ? (long long)g.outC * g.Cg : 0;
  long long wblocks = (std::max(total, gb != nullptr ? (long long)g.outC : 0LL) + 255) / 256;
  if (wblocks > 148LL * 16) wblocks = 148LL * 16;
  if (tiles + wblocks == 0) return cudaSuccess;
  const int tiles_x = transpose4_tiles_x(g.C);
  const int per_img = tiles_x * ((g.HW + 63) / 64);
  const int Ppad = (g.P + 3) & ~3;
  const int pspans = (Ppad + PG_SPAN - 1) / PG_SPAN;
  bwd_finish_kernel<<<(unsigned)(tiles + wblocks), 256, 0, stream>>>(
      gxt, gx, g.C, g.HW, tiles_x, per_img, (int)tiles, gwt, gw, g.Cg, g.kk, total,
      gb != nullptr ? gpart : nullptr, gb, g.N, g.outC, pspans);
  return cudaGetLastError();
}

bool tc_fused_supported(const Geom& g) {
  return tc_bwd_supported(g) && g.Og <= 256 && (long long)g.G * weight_slots(g) *
                                                  (((long long)g.N * ((g.P + 31) / 32) + 3) / 4) <
                                                  (1LL << 40);
}

namespace {
// Grid and schedule of the fused backward, and the launch.
template <int FMT>
cudaError_t launch_fused(const Geom& g, const CUtensorMap& amap, const CUtensorMap& bmap,
                         const CUtensorMap& g2map, const void* xt, const void* off,
                         const void* mask, float* gxt, float* goff, float* gmask, float* gwt,
                         int num_sms, cudaStream_t stream) {
  const size_t smem = fused_smem_bytes();
  cudaError_t e =
      ensure_dynamic_smem(reinterpret_cast<const void*>(bwd_fused_tc_kernel<FMT>), (int)smem);
  if (e != cudaSuccess) return e;
  const int bpi = (g.P + 31) / 32;  // 32-pixel blocks per image
  if ((long long)g.N * bpi > (1LL << 30)) return cudaErrorInvalidValue;
  const int nblocks = g.N * bpi;
  const int mtiles = (nblocks + 3) / 4;
  const int nslots = weight_slots(g);
  const long long slots = (long long)g.G * nslots;
  const long long nitems = slots * mtiles;
  // aligned pixel ranges per slot when the slots fit the SMs (at most one
  // range per tile); else contiguous cuts of the slot-major item list
  int ranges = slots <= num_sms ? (int)(num_sms / slots) : 0;
  if (ranges > mtiles) ranges = mtiles;
  const int grid = ranges > 0 ? (int)(ranges * slots)
                              : (int)(nitems < num_sms ? nitems : num_sms);
  bwd_fused_tc_kernel<FMT><<<grid, F_THREADS, smem, stream>>>(
      g, amap, bmap, g2map, bpi, nblocks, mtiles, nslots, nitems, ranges, xt, off, mask, gxt,
      goff, gmask, gwt);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_bwd_fused_tc(const Geom& g, const float* go_r, const float* wbt,
                                const float* xt, const float* off, const float* mask, float* gxt,
                                float* goff, float* gmask, float* gwt, int num_sms,
                                cudaStream_t stream) {
  if (!tc_fused_supported(g)) return cudaErrorInvalidValue;
  const int Ppad = (g.P + 3) & ~3;
  CUtensorMap amap, bmap, g2map;
  // go_r rows of P pixels: 32-pixel x 32-row boxes (GEMM1's A, MN-major) and
  // 32-pixel x Og-row boxes (GEMM2's B, K-major); pixels past P read as zero
  cudaError_t e = make_tmap_2d_f32(&amap, go_r, (uint64_t)g.P, (uint64_t)g.N * g.outC,
                                   (uint64_t)Ppad, 32u, /*atom32=*/true);
  if (e != cudaSuccess) return e;
  // packed W: rows of (tap, channel), Og out channels each; 128-row boxes
  e = make_tmap_2d_f32(&bmap, wbt, (uint64_t)g.Og, (uint64_t)g.G * g.kk * g.Cg, (uint64_t)g.Og,
                       128u);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d_f32(&g2map, go_r, (uint64_t)g.P, (uint64_t)g.N * g.outC, (uint64_t)Ppad,
                       (uint32_t)g.Og);
  if (e != cudaSuccess) return e;
  return launch_fused<kF32>(g, amap, bmap, g2map, xt, off, mask, gxt, goff, gmask, gwt, num_sms,
                            stream);
}

namespace {
// 16-bit grad_out (N*outC rows of P) -> go_r rows padded to Ppad (a multiple
// of 8: 16-byte pitch; the padding zero), its values unchanged; with `gb`
// (fp32, pre-zeroed) the bias gradient summed on the way in fp32, or with
// `gpart` the span's sum written to gpart[bid] (as prep_go_block).
template <int FMT>
__device__ __forceinline__ void prep_go16_block(long long bid,
                                                const unsigned short* __restrict__ go,
                                                unsigned short* __restrict__ go_r,
                                                float* __restrict__ gb, float* __restrict__ gpart,
                                                int outC, int P, int Ppad, int pspans, int vec) {
  __shared__ float part[8];
  const long long row = bid / pspans;  // n * outC + o
  const int pbeg = (int)(bid - row * pspans) * PG_SPAN;
  const int pend = min(Ppad, pbeg + PG_SPAN);
  const unsigned short* src = go + row * P;
  unsigned short* dst = go_r + row * Ppad;
  float sum = 0.f;
  if (vec) {  // P % 8 == 0: Ppad == P, 16-byte aligned rows, 8 values a load
    for (int p = pbeg + 8 * threadIdx.x; p < pend; p += 8 * blockDim.x) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(src + p));
      *reinterpret_cast<uint4*>(dst + p) = v;
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) sum += h_lo<FMT>(w[e]) + h_hi<FMT>(w[e]);
    }
  } else {
    for (int p = pbeg + threadIdx.x; p < pend; p += blockDim.x) {
      const unsigned short v = p < P ? __ldg(src + p) : (unsigned short)0;
      dst[p] = v;
      if constexpr (FMT == kF16s) sum += __half2float(__ushort_as_half(v));
      else sum += __uint_as_float((uint32_t)v << 16);
    }
  }
  if (gb == nullptr && gpart == nullptr) return;
#pragma unroll
  for (int d = 16; d > 0; d >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, d);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = sum;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += part[w];
    if (gpart != nullptr) gpart[bid] = t;
    else atomicAdd(gb + row % outC, t);
  }
}
template <int FMT>
__global__ void __launch_bounds__(256) prep_go16_kernel(const unsigned short* __restrict__ go,
                                                        unsigned short* __restrict__ go_r,
                                                        float* __restrict__ gb, int outC, int P,
                                                        int Ppad, int pspans, int vec) {
  prep_go16_block<FMT>(blockIdx.x, go, go_r, gb, nullptr, outC, P, Ppad, pspans, vec);
}

// 16-bit weight (outC, Cg, kh, kw) -> wbt[(g*kk + k)*Cg + c][o] (16-bit, as
// the fp32 pack of the grad-column operand): elements [i0, i1), thread t of
// 256 takes i0 + t, i0 + t + stride, ...
__device__ __forceinline__ void pack16_range(long long i0, long long i1, long long stride,
                                             const unsigned short* __restrict__ w,
                                             unsigned short* __restrict__ wb, const Geom& g) {
  for (long long i = i0 + threadIdx.x; i < i1; i += stride) {
    // i enumerates the output: ((gi*kk + k)*Cg + c)*Og + o
    const int o = (int)(i % g.Og);
    long long r = i / g.Og;
    const int c = (int)(r % g.Cg);
    r /= g.Cg;
    const int k = (int)(r % g.kk);
    const int gi = (int)(r / g.kk);
    wb[i] = __ldg(w + ((long long)(gi * g.Og + o) * g.Cg + c) * g.kk + k);
  }
}
__global__ void __launch_bounds__(256) pack_weight_bwd16_kernel(
    const unsigned short* __restrict__ w, unsigned short* __restrict__ wb, Geom g,
    long long total) {
  pack16_range(blockIdx.x * 256LL, total, (long long)gridDim.x * 256, w, wb, g);
}

// The 16-bit fused backward's helpers in one launch, as bwd_prologue_kernel:
// items [0, nb_prep) prepare a grad_out span each (grad_bias partial sums),
// the next nb_pack pack PACK16_ITEM weight elements each, the rest zero the
// accumulators.
constexpr int PACK16_ITEM = 2048;
struct Prologue16 {
  const unsigned short* go;
  unsigned short* go_r;
  float* gpart;
  const unsigned short* w;
  unsigned short* wbt;
  long long wtotal;
  ZeroItems z;
  int Ppad, pspans, vec;
  int nb_prep, nb_pack, total;
};
template <int FMT>
__global__ void __launch_bounds__(256) bwd_prologue16_kernel(Prologue16 a, Geom g) {
  for (int it = blockIdx.x; it < a.total; it += gridDim.x) {
    int b = it;
    if (b < a.nb_prep) {
      prep_go16_block<FMT>(b, a.go, a.go_r, nullptr, a.gpart, g.outC, g.P, a.Ppad, a.pspans,
                           a.vec);
    } else if ((b -= a.nb_prep) < a.nb_pack) {
      const long long i0 = (long long)b * PACK16_ITEM;
      pack16_range(i0, std::min<long long>(i0 + PACK16_ITEM, a.wtotal), 256, a.w, a.wbt, g);
    } else {
      zero_item(a.z, b - a.nb_pack);
    }
    __syncthreads();  // the shared staging of one item is free before the next
  }
}

// fp32 NHWC (N, HW, C) -> 16-bit NCHW (N, C, HW), rounded to nearest; 32x32
// tiles.
template <int FMT>
__global__ void __launch_bounds__(256) nhwc_to_nchw16_kernel(const float* __restrict__ in,
                                                             unsigned short* __restrict__ out,
                                                             int HW, int C) {
  __shared__ float tile[32][33];
  const int n = blockIdx.z;
  const int p0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
  const float* src = in + (long long)n * HW * C;
  unsigned short* dst = out + (long long)n * HW * C;
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int p = p0 + ty + i, c = c0 + tx;
    if (p < HW && c < C) tile[ty + i][tx] = src[(long long)p * C + c];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int c = c0 + ty + i, p = p0 + tx;
    if (p < HW && c < C) {
      const float v = tile[tx][ty + i];
      if constexpr (FMT == kF16s) dst[(long long)c * HW + p] = __half_as_ushort(__float2half_rn(v));
      else dst[(long long)c * HW + p] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
  }
}

// The 16-bit backward's gradients in one launch: the tap-major fp32 weight
// gradient gwt[o][k][c] to grad_weight[o][c][k], then up to three fp32
// arrays element-wise (grad_offset, grad_mask, grad_bias), all rounded to 16
// bits (to nearest even).  One index space over all of them, grid-stride.
template <int FMT>
__global__ void __launch_bounds__(256) grads_to_h16_kernel(const float* __restrict__ gwt,
                                                           unsigned short* __restrict__ gw,
                                                           int Cg, int kk, long long nw,
                                                           H16List rest,
                                                           const float* __restrict__ gpart,
                                                           unsigned short* __restrict__ gb16,
                                                           int N, int outC, int pspans) {
  if (gpart != nullptr)  // grad_bias from the prologue's partial sums, in a fixed order
    for (long long o = blockIdx.x * 256LL + threadIdx.x; o < outC; o += gridDim.x * 256LL) {
      float t = 0.f;
      for (int n = 0; n < N; ++n)
        for (int sp = 0; sp < pspans; ++sp)
          t += __ldg(gpart + ((long long)n * outC + o) * pspans + sp);
      if constexpr (FMT == kF16s) gb16[o] = __half_as_ushort(__float2half_rn(t));
      else gb16[o] = __bfloat16_as_ushort(__float2bfloat16_rn(t));
    }
  const long long total = nw + rest.n[0] + rest.n[1] + rest.n[2];
  for (long long i = blockIdx.x * 256LL + threadIdx.x; i < total; i += (long long)gridDim.x * 256) {
    float v;
    unsigned short* dst;
    if (i < nw) {  // i = (o*Cg + c)*kk + k
      const long long ock = (long long)Cg * kk;
      const long long o = i / ock;
      const int r = (int)(i - o * ock);
      const int c = r / kk, k = r - c * kk;
      v = __ldg(gwt + o * ock + (long long)k * Cg + c);
      dst = gw + i;
    } else {
      long long j = i - nw;
      int a = 0;
      while (a < 2 && j >= rest.n[a]) j -= rest.n[a++];
      v = __ldg(rest.src[a] + j);
      dst = rest.dst[a] + j;
    }
    if constexpr (FMT == kF16s) *dst = __half_as_ushort(__float2half_rn(v));
    else *dst = __bfloat16_as_ushort(__float2bfloat16_rn(v));
  }
}
}  // namespace

cudaError_t launch_grads_to_h16(const float* gwt, void* gw, const Geom& g, const H16List& rest,
                                bool f16, cudaStream_t stream, const float* gpart, void* gb) {
  const long long nw = (long long)g.outC * g.Cg * g.kk;
  const long long total = nw + rest.n[0] + rest.n[1] + rest.n[2] + (gpart ? g.outC : 0);
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 8) blocks = 148LL * 8;
  const int Ppad = (g.P + 7) & ~7;
  auto kern = f16 ? grads_to_h16_kernel<kF16s> : grads_to_h16_kernel<kBF16s>;
  kern<<<(int)blocks, 256, 0, stream>>>(gwt, static_cast<unsigned short*>(gw), g.Cg, g.kk, nw,
                                        rest, gb != nullptr ? gpart : nullptr,
                                        static_cast<unsigned short*>(gb), g.N, g.outC,
                                        (Ppad + PG_SPAN - 1) / PG_SPAN);
  return cudaGetLastError();
}

cudaError_t launch_prep_go16(const Geom& g, const void* go, void* go_r, float* gb, bool f16,
                             cudaStream_t stream) {
  if ((long long)g.N * g.outC * g.P == 0) return cudaSuccess;
  const int Ppad = (g.P + 7) & ~7;
  const int pspans = (Ppad + PG_SPAN - 1) / PG_SPAN;
  const long long blocks = (long long)g.N * g.outC * pspans;
  if (blocks > (1LL << 31) - 1) return cudaErrorInvalidValue;
  const int vec = g.P % 8 == 0 && (reinterpret_cast<uintptr_t>(go) & 15u) == 0 &&
                  (reinterpret_cast<uintptr_t>(go_r) & 15u) == 0;
  auto kern = f16 ? prep_go16_kernel<kF16s> : prep_go16_kernel<kBF16s>;
  kern<<<(unsigned)blocks, 256, 0, stream>>>(static_cast<const unsigned short*>(go),
                                              static_cast<unsigned short*>(go_r), gb, g.outC,
                                              g.P, Ppad, pspans, vec);
  return cudaGetLastError();
}

cudaError_t launch_pack_weight_bwd16(const void* w, void* wbt, const Geom& g,
                                     cudaStream_t stream) {
  const long long total = (long long)g.G * g.kk * g.Cg * g.Og;
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148LL * 16) blocks = 148LL * 16;
  pack_weight_bwd16_kernel<<<(int)blocks, 256, 0, stream>>>(
      static_cast<const unsigned short*>(w), static_cast<unsigned short*>(wbt), g, total);
  return cudaGetLastError();
}

cudaError_t launch_bwd_prologue16(const Geom& g, const void* go, void* go_r, float* gpart,
                                  const void* w, void* wbt, const ZeroList& z, bool f16,
                                  cudaStream_t stream) {
  if (g.P == 0 || z.count > 4) return cudaErrorInvalidValue;
  Prologue16 a{};
  a.go = static_cast<const unsigned short*>(go);
  a.go_r = static_cast<unsigned short*>(go_r);
  a.gpart = gpart;
  a.w = static_cast<const unsigned short*>(w);
  a.wbt = static_cast<unsigned short*>(wbt);
  a.wtotal = (long long)g.G * g.kk * g.Cg * g.Og;
  if (!zero_items(z, a.z)) return cudaErrorInvalidValue;
  a.Ppad = (g.P + 7) & ~7;
  a.pspans = (a.Ppad + PG_SPAN - 1) / PG_SPAN;
  a.vec = g.P % 8 == 0 && (reinterpret_cast<uintptr_t>(go) & 15u) == 0 &&
          (reinterpret_cast<uintptr_t>(go_r) & 15u) == 0;
  const long long prep = (long long)g.N * g.outC * a.pspans;
  const long long pack = (a.wtotal + PACK16_ITEM - 1) / PACK16_ITEM;
  const long long total = prep + pack + a.z.total;
  if (total > (1LL << 31) - 1) return cudaErrorInvalidValue;
  a.nb_prep = (int)prep;
  a.nb_pack = (int)pack;
  a.total = (int)total;
  const long long grid = std::min<long long>(total, (long long)device_sm_count() * 8);
  auto kern = f16 ? bwd_prologue16_kernel<kF16s> : bwd_prologue16_kernel<kBF16s>;
  kern<<<(unsigned)grid, 256, 0, stream>>>(a, g);
  return cudaGetLastError();
}

size_t tc_bias_part_floats16(const Geom& g) {
  const int Ppad = (g.P + 7) & ~7;
  return (size_t)g.N * g.outC * ((Ppad + PG_SPAN - 1) / PG_SPAN);
}

cudaError_t launch_nhwc_to_nchw16(const float* gxt, void* gx, int N, int C, int HW, bool f16,
                                  cudaStream_t stream) {
  if ((long long)N * C * HW == 0) return cudaSuccess;
  if (N > 65535 || (HW + 31) / 32 > 65535) return cudaErrorInvalidValue;
  dim3 grid((C + 31) / 32, (HW + 31) / 32, N);
  auto kern = f16 ? nhwc_to_nchw16_kernel<kF16s> : nhwc_to_nchw16_kernel<kBF16s>;
  kern<<<grid, 256, 0, stream>>>(gxt, static_cast<unsigned short*>(gx), HW, C);
  return cudaGetLastError();
}

bool tc_fused16_supported(const Geom& g) { return tc_fused_supported(g) && g.C % 8 == 0; }

cudaError_t launch_bwd_fused_tc_h16(const Geom& g, const void* go_r, const void* wbt,
                                    const void* xt, const void* off, const void* mask,
                                    float* gxt, float* goff, float* gmask, float* gwt, bool f16,
                                    int num_sms, cudaStream_t stream) {
  if (!tc_fused16_supported(g)) return cudaErrorInvalidValue;
  const int Ppad = (g.P + 7) & ~7;  // 16-byte row pitch
  CUtensorMap amap, bmap, g2map;
  // go_r rows: 32-pixel x 64-row boxes, 64-byte swizzle (GEMM1's A, MN-major)
  // and 32-pixel x Og-row boxes, 64-byte swizzle (GEMM2's B, K-major)
  cudaError_t e = make_tmap_2d_h16_box(&amap, go_r, (uint64_t)g.P, (uint64_t)g.N * g.outC,
                                       (uint64_t)Ppad, 32u, 64u, f16);
  if (e != cudaSuccess) return e;
  // packed W: 64-out-channel x 128-row boxes, 128-byte swizzle (K-major)
  e = make_tmap_2d_h16_box(&bmap, wbt, (uint64_t)g.Og, (uint64_t)g.G * g.kk * g.Cg,
                           (uint64_t)g.Og, 64u, 128u, f16);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d_h16_box(&g2map, go_r, (uint64_t)g.P, (uint64_t)g.N * g.outC, (uint64_t)Ppad,
                           32u, (uint32_t)g.Og, f16);
  if (e != cudaSuccess) return e;
  return f16 ? launch_fused<kF16s>(g, amap, bmap, g2map, xt, off, mask, gxt, goff, gmask, gwt,
                                   num_sms, stream)
             : launch_fused<kBF16s>(g, amap, bmap, g2map, xt, off, mask, gxt, goff, gmask, gwt,
                                    num_sms, stream);
}

bool tc_wcol_supported(const Geom& g, bool split) {
  return tc_bwd_supported(g) && (long long)g.kk * g.NP * (split ? 2 : 1) < (1LL << 31);
}

size_t tc_col_bytes(const Geom& g, bool split) {
  return (size_t)(split ? 2 : 1) * g.kk * g.NP * g.C * sizeof(float);
}

cudaError_t launch_bwd_weight_col(const Geom& g, const float* col, const float* go_r, float* gw,
                                  bool tap_major, bool split, int num_sms, cudaStream_t stream) {
  if (!tc_wcol_supported(g, split)) return cudaErrorInvalidValue;
  const int bn = weight_bn(g);
  const int Ppad = (g.P + 3) & ~3;
  CUtensorMap colmap, gomap;
  cudaError_t e = make_tmap_2d_f32(&colmap, col, (uint64_t)g.C,
                                   (uint64_t)g.kk * g.NP * (split ? 2 : 1), (uint64_t)g.C, 32u,
                                   /*atom32=*/true);
  if (e != cudaSuccess) return e;
  e = make_tmap_2d_f32(&gomap, go_r, (uint64_t)Ppad, (uint64_t)g.N * g.outC * (split ? 2 : 1),
                       (uint64_t)Ppad, (uint32_t)bn);
  if (e != cudaSuccess) return e;
  const size_t smem = weight_smem_bytes(bn, split);
  auto kern = split ? bwd_weight_col_kernel<true> : bwd_weight_col_kernel<false>;
  e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem);
  if (e != cudaSuccess) return e;
  const WSplit w = weight_split(g, bn, num_sms, 16);
  if (w.ntiles > (1LL << 30)) return cudaErrorInvalidValue;
  const int grid = (int)(w.ntiles < num_sms ? w.ntiles : num_sms);
  kern<<<grid, WC_THREADS, smem, stream>>>(g, colmap, gomap, bn, pow2_cols(2 * bn), gw,
                                            tap_major ? g.Cg : 1, tap_major ? 1 : g.kk,
                                            weight_slots(g), w.ntn, w.splits, w.per,
                                            (int)w.ntiles);
  return cudaGetLastError();
}

}  // namespace dcn
