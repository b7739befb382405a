// dcn_fwd_tc.cu -- forward deformable convolution on the 5th-generation
// tensor cores (tcgen05, kind::tf32, fp32 accumulation in tensor memory).
//
// Implicit GEMM per group g:  D[pixels, out channels] = A . B^T with
//   A[q, (k, c)] = mask * bilinear(x[n, c], sample(q, k))   (deform_conv2d.metal:74-125)
//   B[o, (k, c)] = W[g*Og + o, c, k]
// K ordered (tap, channel); a K step is 32 channels of one tap (128 bytes of
// tf32 per row, one 128-byte swizzle row).  The column matrix A never touches
// HBM.
//
// Persistent, warp-specialised CTA (one per SM), tiles of 128 pixels x BN out
// channels handed out round-robin:
//   warps 0-3   epilogue: tcgen05.ld of a finished accumulator, + bias,
//               NCHW stores; overlaps the next tile's main loop
//   warp  4     MMA issue (one thread): 4 UMMAs of 128 x BN x 8 per K step
//   warp  5     TMA producer of the weight tile (BN rows x 128 B per K step)
//   warps 6-21  16 gather warps: each owns 8 pixel rows of A, computes the
//               bilinear sampling plan once per (tap, deformable group), and
//               per K step issues its 8 corner loads (16 B, NHWC input),
//               combines, rounds to TF32 and stores into the swizzled stage
// A 4-stage shared-memory ring (A 16 KB + B up to 32 KB per stage) is guarded
// by mbarriers: full[s] = 16 gather-warp arrivals, tfull[s] = the weight
// tile's TMA transaction bytes; empty[s] = tcgen05.commit of the MMAs that
// read it.  Two accumulators of BN columns in tensor memory (acc_full /
// acc_empty barriers) let the epilogue of tile i run while tile i+1 is being
// accumulated.  Every wait is bounded (tc::Watch): the first one that runs
// out raises bit 1 of g_tc_fwd_status and makes every role of the CTA leave.
//
// 3xTF32 (SPLIT): each operand is carried as a high TF32 part and a low TF32
// part (x - hi); every K step issues lo.hi + hi.lo + hi.hi, which recovers
// fp32-level products at three times the tensor work (2 stages of twice the
// size instead of 4).
//
// The packed weight is rounded to TF32 with round-to-nearest; the gathered
// column values are staged as fp32 and the tensor core uses their TF32 part
// (the low 13 mantissa bits are ignored), a relative error below 2^-10 per
// value -- well inside the output tolerance of TF32 mode.  The backward kernels
// round their gathered operands to nearest, as the gradients have the tighter
// tolerance.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "dcn_launch.h"
#include "dcn_tc.h"
#include "dcn_tc_common.cuh"
#include "dcn_tma.h"
#include "dcn_transpose.cuh"

namespace dcn {

// Error word of the tensor-core forward: bit 1 is raised by a wait that ran
// out (read and cleared by read_fwd_status).
__device__ int g_tc_fwd_status;

namespace {

constexpr int BM = 128;
constexpr int GATHER_WARPS = 16;
constexpr int EPI_WARPS = 4;
constexpr int MMA_WARP = 4, TMA_WARP = 5, GATHER_WARP0 = 6;
constexpr int THREADS = (GATHER_WARP0 + GATHER_WARPS) * 32;  // 704
constexpr int A_STAGE = BM * 128;                            // 16 KB

int tc_bn(const Geom& g) { return g.Og <= 256 ? g.Og : 256; }
int tmem_cols_for(int bn) {
  int c = 32;
  while (c < 2 * bn) c <<= 1;
  return c;
}
// Operand modes of the kernel:
//   TF32   fp32 tensors, TF32 operands (A staged as fp32, read as TF32);
//   SPLIT  3xTF32: high and low TF32 parts of each operand, three UMMAs per
//          K substep, twice the stage bytes so half the stages;
//   BF16   bf16 tensors (NHWC copy, packed weight, offsets, mask, bias and
//          output all bf16), kind::f16 UMMAs with bf16 operands; a K step is
//          64 channels (still 128 B per row) and each gather lane blends 16;
//   F16    the same with fp16 tensors and fp16 operands.
enum : int { kTF32 = 0, kSplit = 1, kBF16 = 2, kF16 = 3 };
// Storage formats of the small operands and of the output.
enum : int { kFmtF32 = 0, kFmtBF16 = 1, kFmtF16 = 2 };
template <int MODE>
struct FwdCfg {
  static constexpr bool SPLIT = MODE == kSplit;
  static constexpr bool H16 = MODE == kBF16 || MODE == kF16;  // 16-bit storage
  static constexpr int FMT = MODE == kBF16 ? kFmtBF16 : (MODE == kF16 ? kFmtF16 : kFmtF32);
  static constexpr int STAGES = SPLIT ? 2 : 4;
  static constexpr int PARTS = SPLIT ? 2 : 1;
  static constexpr int KCH = H16 ? 64 : 32;  // channels of one tap per K step
};
// Barriers and flags after the stage ring: full, tfull, empty (one per stage),
// acc_full, acc_empty (two), drain, then the tensor-memory address and the
// abort flag.
constexpr int kBarrierBytes = 256;
size_t smem_bytes(int bn, bool split) {
  const int parts = split ? 2 : 1, stages = split ? 2 : 4;
  return (size_t)stages * parts * (A_STAGE + (size_t)bn * 128) + kBarrierBytes + 1024;
}

struct Tile {
  long long q0;
  int o0, gi;
};
__device__ __forceinline__ Tile tile_of(int t, int mtiles, int ntiles_n, int bn) {
  Tile T;
  const int mt = t % mtiles;
  const int r = t / mtiles;
  T.q0 = (long long)mt * BM;
  T.o0 = (r % ntiles_n) * bn;
  T.gi = r / ntiles_n;
  return T;
}

// Schedule of a launch.  Tiles [0, whole) go round-robin over the grid, one
// CTA each.  When the tile count leaves the last round short (tiles % grid SMs
// busy, most of them idle), the remaining tiles are split by K instead: their K
// steps, laid end to end, are cut into `ctas` equal ranges, one per CTA, so
// every CTA runs about the same number of K steps.  A range covers the end of
// one tile and the start of the next at most; each piece of a tile leaves its
// partial sum in a slot (2 per CTA, [tn][BM] floats), and fwd_tail_sum_kernel,
// launched after the forward, adds every split tile's pieces in CTA order --
// a fixed order, so the output does not depend on which piece finishes first
// -- with all of the GPU's threads on it.  No CTA waits for another.
struct TailPlan {
  int whole;               // tiles handed out whole
  int ctas;                // CTAs sharing the split tiles (0: no split)
  long long tail_steps;    // K steps of the split tiles
  float* part;             // partial slots
};
struct Work {
  int t;       // tile
  int s0, s1;  // its K steps [s0, s1)
  int slot;    // partial slot, -1 for a whole tile
};
// Runs f(work) for this CTA's work in order: its whole tiles, then its pieces
// of split tiles, until f returns false (a wait of the CTA gave up).  The two
// loops inline f separately, so the whole-tile loop keeps no split state live.
template <class F>
__device__ __forceinline__ void for_each_work(const TailPlan& tp, int steps, F&& f) {
  for (int t = blockIdx.x; t < tp.whole; t += gridDim.x)
    if (!f(Work{t, 0, steps, -1})) return;
  if ((int)blockIdx.x >= tp.ctas) return;
  // tail_steps < 2^30 (host), so the positions fit in int
  int x = (int)((long long)blockIdx.x * tp.tail_steps / tp.ctas);
  const int xend = (int)((long long)(blockIdx.x + 1) * tp.tail_steps / tp.ctas);
  for (int seg = 0; x < xend; ++seg) {
    const int j = x / steps;
    const int s0 = x - j * steps;
    const int s1 = xend - x < steps - s0 ? s0 + (xend - x) : steps;
    if (!f(Work{tp.whole + j, s0, s1, 2 * (int)blockIdx.x + seg})) return;
    x += s1 - s0;
  }
}
// CTA whose K range holds split step x: the largest c with c*T/ctas <= x.
__device__ __forceinline__ int tail_cta_of(const TailPlan& tp, long long x) {
  return (int)(((x + 1) * tp.ctas - 1) / tp.tail_steps);
}

// Scalar loads of the small operands (offsets, mask, bias) as fp32.
template <int FMT>
__device__ __forceinline__ float ld_io(const void* p, long long i) {
  if constexpr (FMT == kFmtBF16) {
    const unsigned short v = __ldg(reinterpret_cast<const unsigned short*>(p) + i);
    return __uint_as_float((uint32_t)v << 16);
  } else if constexpr (FMT == kFmtF16) {
    return __half2float(__ldg(reinterpret_cast<const __half*>(p) + i));
  } else {
    return __ldg(reinterpret_cast<const float*>(p) + i);
  }
}
// 256-bit global load (sm_100): 32 bytes at a 32-byte aligned address.
__device__ __forceinline__ void ldg_v8(const void* p, uint32_t (&r)[8]) {
  asm volatile("ld.global.nc.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                 "=r"(r[6]), "=r"(r[7])
               : "l"(p));
}
__device__ __forceinline__ void st_shared_u4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c,
                                             uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}
// The two 16-bit values of a 32-bit word (low half first) as fp32, and back.
template <int FMT>
__device__ __forceinline__ float h16_lo(uint32_t w) {
  if constexpr (FMT == kFmtF16) return __half2float(__ushort_as_half((unsigned short)(w & 0xffffu)));
  else return __uint_as_float(w << 16);
}
template <int FMT>
__device__ __forceinline__ float h16_hi(uint32_t w) {
  if constexpr (FMT == kFmtF16) return __half2float(__ushort_as_half((unsigned short)(w >> 16)));
  else return __uint_as_float(w & 0xffff0000u);
}
template <int FMT>
__device__ __forceinline__ uint32_t pack_h16x2(float lo, float hi) {
  if constexpr (FMT == kFmtF16) {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}
template <int FMT>
__device__ __forceinline__ unsigned short to_h16(float y) {
  if constexpr (FMT == kFmtF16) return __half_as_ushort(__float2half_rn(y));
  else return __bfloat16_as_ushort(__float2bfloat16_rn(y));
}

// 704 threads: 22 warps, up to 6 on one SM sub-partition of 16K registers,
// so at most 80 registers a thread (a few bytes spill).
// NH = 2: tiles of 2 x 256 out channels (out channels per group a multiple of
// 512): the gathered A tile feeds both halves, so it is gathered once instead
// of once per 256 out channels; the two accumulators fill tensor memory (no
// double buffering) and 80 KB stages leave room for two.
template <int MODE, int NH>
__global__ void __launch_bounds__(THREADS, 1)
fwd_tc_kernel(Geom g, const __grid_constant__ CUtensorMap wmap, const void* __restrict__ xt_,
              int bn, int tcols, int mtiles, int ntiles_n, TailPlan tp,
              const void* __restrict__ off, const void* __restrict__ mask,
              const void* __restrict__ bias, void* __restrict__ out) {
  using Cfg = FwdCfg<MODE>;
  constexpr bool SPLIT = Cfg::SPLIT, H16 = Cfg::H16;
  constexpr int FMT = Cfg::FMT;
  constexpr int STAGES = NH == 2 ? 2 : Cfg::STAGES, PARTS = Cfg::PARTS, KCH = Cfg::KCH;
  static_assert(NH == 1 || (NH == 2 && !SPLIT), "wide tiles for single-part operands");
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw_u32 & 1023u)) & 1023u);
  const uint32_t sA0 = tc::smem_u32(smem);
  const int tn = NH * bn;  // out channels of a tile
  const uint32_t b_stage = (uint32_t)tn * 128;
  const uint32_t sB0 = sA0 + STAGES * PARTS * A_STAGE;
  // full[s]: the 16 gather warps' A rows; tfull[s]: the weight tile's TMA
  // bytes (a barrier of its own, so the TMA warp can drain its copies alone)
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * PARTS * (A_STAGE + b_stage));
  uint64_t* tfull = full + STAGES;
  uint64_t* empty = tfull + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  const tc::Watch watch{abort_flag, &g_tc_fwd_status, kStatusFwd, g.wait_limit};

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nchunk = g.Cg / KCH;
  const int steps = g.kk * nchunk;

  if (tid == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], GATHER_WARPS);
      tc::mbar_init(&tfull[s], 1);
      tc::mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(&acc_full[a], 1);
      tc::mbar_init(&acc_empty[a], EPI_WARPS);
    }
    tc::mbar_init(drain, 1);
    *abort_flag = 0;
    tc::fence_mbar_init();
  }
  if (warp == MMA_WARP) {
    tc::tmem_alloc(tmem_slot, (uint32_t)tcols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp >= GATHER_WARP0) {
    // ------------------------------ gather ------------------------------
    // Dropped corners read the zero pixel row that follows the NHWC copy, so
    // the corner loads are unconditional.  A warp owns 8 pixel rows of the
    // tile; 4 lanes share a row, each loading a 32-byte run of it per corner
    // (one 256-bit load: 8 fp32 or 16 bf16 channels) and storing two 16-byte
    // chunks of the swizzled row.
    const int gw = warp - GATHER_WARP0;
    const int q4 = lane & 3, sub = lane >> 2;
    const int zoff = g.N * g.HW * g.C;  // element offset of the zero row
    const char* xq = static_cast<const char*>(xt_) + q4 * 32;
    constexpr int ESZ = H16 ? 2 : 4;  // element bytes
    int gs = 0;
    for_each_work(tp, steps, [&](const Work& w) {
      const Tile T = tile_of(w.t, mtiles, ntiles_n, tn);
      const int row = gw * 8 + sub;
      const long long q = T.q0 + row;
      const bool rvalid = q < g.NP;
      const int rn = rvalid ? (int)(q / g.P) : 0;
      const int rp = rvalid ? (int)(q - (long long)rn * g.P) : 0;
      const int roy = rp / g.Wo, rox = rp - roy * g.Wo;
      const uint32_t soff0 = tc::sw128_offset(row, 2 * q4), soff1 = tc::sw128_offset(row, 2 * q4 + 1);
      int coff[4];  // element offsets of the corners' channel vectors
      float cw[4];
      // incremental (tap, channel chunk, deformable group) counters, from
      // K step s0 = k * nchunk + c0 / KCH
      int k = w.s0 / nchunk, c0 = (w.s0 - k * nchunk) * KCH;
      int ki = k / g.kw, kj = k - ki * g.kw;
      const int gbase = T.gi * g.Cg;
      int dgi = (gbase + c0) / g.cpg, cpos = gbase + c0 - dgi * g.cpg;
      bool replan = true;
      for (int s = w.s0; s < w.s1; ++s, ++gs) {
        const int st = gs % STAGES;
        const int u = gs / STAGES;
        if (replan) {
          replan = false;
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            coff[c] = zoff;
            cw[c] = 0.f;
          }
          if (rvalid) {
            const long long oi = off_h_index(g, rn, dgi, k, rp);
            const float h = (float)((roy + g.oy0) * g.sh - g.ph + ki * g.dh) + ld_io<FMT>(off, oi);
            const float w = (float)(rox * g.sw - g.pw + kj * g.dw) + ld_io<FMT>(off, oi + g.P);
            float m = 1.f;
            if (g.use_mask) {
              const float raw = ld_io<FMT>(mask, mask_index(g, rn, dgi, k, rp));
              m = g.mask_logits ? 1.f / (1.f + expf(-raw)) : raw;
            }
            const Sample sp = make_sample(h, w, g.H, g.W);
            if (sp.valid) {
              const int xn = rn * g.HW;
              if (sp.live & 1u) { coff[0] = (xn + sp.i1) * g.C; cw[0] = sp.w1 * m; }
              if (sp.live & 2u) { coff[1] = (xn + sp.i2) * g.C; cw[1] = sp.w2 * m; }
              if (sp.live & 4u) { coff[2] = (xn + sp.i3) * g.C; cw[2] = sp.w3 * m; }
              if (sp.live & 8u) { coff[3] = (xn + sp.i4) * g.C; cw[3] = sp.w4 * m; }
            }
          }
        }
        // issue the loads before waiting for the stage to be free
        const int gch0 = gbase + c0;
        const uint32_t sA = sA0 + st * PARTS * A_STAGE;
        uint32_t v[4][8];
#pragma unroll
        for (int c = 0; c < 4; ++c)
          ldg_v8(xq + (size_t)(unsigned)(coff[c] + gch0) * ESZ, v[c]);
        if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return false;
        const float a = cw[0], b = cw[1], c = cw[2], d = cw[3];
        if constexpr (H16) {
          uint32_t r[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float lo = a * h16_lo<FMT>(v[0][j]) + b * h16_lo<FMT>(v[1][j]) +
                             c * h16_lo<FMT>(v[2][j]) + d * h16_lo<FMT>(v[3][j]);
            const float hi = a * h16_hi<FMT>(v[0][j]) + b * h16_hi<FMT>(v[1][j]) +
                             c * h16_hi<FMT>(v[2][j]) + d * h16_hi<FMT>(v[3][j]);
            r[j] = pack_h16x2<FMT>(lo, hi);
          }
          st_shared_u4(sA + soff0, r[0], r[1], r[2], r[3]);
          st_shared_u4(sA + soff1, r[4], r[5], r[6], r[7]);
        } else {
          float e[8];
#pragma unroll
          for (int j = 0; j < 8; ++j)
            e[j] = a * __uint_as_float(v[0][j]) + b * __uint_as_float(v[1][j]) +
                   c * __uint_as_float(v[2][j]) + d * __uint_as_float(v[3][j]);
          if constexpr (SPLIT) {
            float h[8], l[8];
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              h[j] = tc::to_tf32(e[j]);
              l[j] = tc::to_tf32(e[j] - h[j]);
            }
            tc::st_shared_v4(sA + soff0, h[0], h[1], h[2], h[3]);
            tc::st_shared_v4(sA + soff1, h[4], h[5], h[6], h[7]);
            tc::st_shared_v4(sA + A_STAGE + soff0, l[0], l[1], l[2], l[3]);
            tc::st_shared_v4(sA + A_STAGE + soff1, l[4], l[5], l[6], l[7]);
          } else {
            // stored as fp32; the tensor core reads the TF32 part of each value
            tc::st_shared_v4(sA + soff0, e[0], e[1], e[2], e[3]);
            tc::st_shared_v4(sA + soff1, e[4], e[5], e[6], e[7]);
          }
        }
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&full[st]);
        // advance (tap, chunk, deformable group)
        c0 += KCH;
        cpos += KCH;
        if (cpos == g.cpg) {
          cpos = 0;
          ++dgi;
          replan = true;
        }
        if (c0 == g.Cg) {
          c0 = 0;
          ++k;
          if (++kj == g.kw) {
            kj = 0;
            ++ki;
          }
          dgi = gbase / g.cpg;
          cpos = gbase - dgi * g.cpg;
          replan = true;
        }
      }
      return true;
    });
  } else if (warp == TMA_WARP) {
    // ------------------------------ weights (TMA) ------------------------------
    if (lane == 0 && !g.no_async) {
      int gs = 0;  // stages filled so far
      for_each_work(tp, steps, [&](const Work& w) {
        const Tile T = tile_of(w.t, mtiles, ntiles_n, tn);
        const int row = T.gi * g.Og + T.o0;
        for (int s = w.s0; s < w.s1; ++s, ++gs) {
          const int st = gs % STAGES;
          const int u = gs / STAGES;
          if (u > 0 && !tc::wait(watch, &empty[st], (u - 1) & 1)) return false;
          tc::mbar_arrive_expect_tx(&tfull[st], PARTS * b_stage);
          const uint32_t sB = sB0 + st * PARTS * b_stage;
#pragma unroll
          for (int h = 0; h < NH; ++h)  // 256-row boxes
            tc::tma_load_2d(sB + h * bn * 128, &wmap, s * KCH, row + h * bn, &tfull[st]);
          if constexpr (SPLIT)  // low parts: rows outC .. 2*outC - 1 of the packed weight
            tc::tma_load_2d(sB + b_stage, &wmap, s * KCH, g.outC + row, &tfull[st]);
        }
        return true;
      });
      if (tc::aborted(watch))  // the copies of the last STAGES fills land before exit
        for (int i = gs > STAGES ? gs - STAGES : 0; i < gs; ++i)
          tc::drain_wait(&tfull[i % STAGES], (i / STAGES) & 1, g.wait_limit);
    }
    __syncwarp();
  } else if (warp == MMA_WARP) {
    // ------------------------------ MMA ------------------------------
    if (lane == 0) {
      const uint32_t idesc = FMT == kFmtF16    ? tc::idesc_f16(BM, bn)
                             : FMT == kFmtBF16 ? tc::idesc_bf16(BM, bn)
                                               : tc::idesc_tf32(BM, bn);
      int gs = 0, it = 0;
      for_each_work(tp, steps, [&](const Work& w) {
        // one accumulator set per tile: two alternate (NH = 1), or one fills
        // tensor memory (NH = 2)
        const int acc = NH == 2 ? 0 : (it & 1);
        const int use = NH == 2 ? it : (it >> 1);  // earlier tiles in this accumulator
        if (use >= 1 && !tc::wait(watch, &acc_empty[acc], (use - 1) & 1)) return false;
        tc::tc_fence_after();
        const uint32_t d0 = tmem + (uint32_t)(acc * tn);
        for (int s = w.s0; s < w.s1; ++s, ++gs) {
          const int st = gs % STAGES;
          const uint32_t accum = s != w.s0 ? 1u : 0u;  // the first K step overwrites
          if (!tc::wait(watch, &full[st], (gs / STAGES) & 1) ||
              !tc::wait(watch, &tfull[st], (gs / STAGES) & 1))
            return false;
          tc::tc_fence_after();
          const uint32_t sA = sA0 + st * PARTS * A_STAGE, sB0s = sB0 + st * PARTS * b_stage;
#pragma unroll
          for (int h = 0; h < NH; ++h) {
          const uint32_t d = d0 + (uint32_t)(h * bn), sB = sB0s + (uint32_t)(h * bn * 128);
#pragma unroll
          for (int j = 0; j < 4; ++j) {  // 32 bytes of K per UMMA: 8 tf32 or 16 bf16
            if constexpr (H16) {
              tc::umma_bf16(d, tc::sdesc_sw128(sA + j * 32), tc::sdesc_sw128(sB + j * 32), idesc,
                            accum | (j != 0 ? 1u : 0u));
            } else if constexpr (SPLIT) {  // lo x hi + hi x lo + hi x hi
              tc::umma_tf32(d, tc::sdesc_sw128(sA + A_STAGE + j * 32),
                            tc::sdesc_sw128(sB + j * 32), idesc, accum | (j != 0 ? 1u : 0u));
              tc::umma_tf32(d, tc::sdesc_sw128(sA + j * 32),
                            tc::sdesc_sw128(sB + b_stage + j * 32), idesc, 1u);
              tc::umma_tf32(d, tc::sdesc_sw128(sA + j * 32), tc::sdesc_sw128(sB + j * 32), idesc,
                            1u);
            } else {
              tc::umma_tf32(d, tc::sdesc_sw128(sA + j * 32), tc::sdesc_sw128(sB + j * 32), idesc,
                            accum | (j != 0 ? 1u : 0u));
            }
          }
          }
          tc::umma_commit(&empty[st]);
        }
        tc::umma_commit(&acc_full[acc]);
        ++it;
        return true;
      });
      if (tc::aborted(watch)) {  // every UMMA issued so far completes before exit
        tc::umma_commit(drain);
        tc::drain_wait(drain, 0, g.wait_limit);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ------------------------------
    int it = 0;
    const int r = warp * 32 + lane;
    for_each_work(tp, steps, [&](const Work& w) {
      const Tile T = tile_of(w.t, mtiles, ntiles_n, tn);
      const int i = it++;
      const int acc = NH == 2 ? 0 : (i & 1);
      if (!tc::wait(watch, &acc_full[acc], (NH == 2 ? i : (i >> 1)) & 1)) return false;
      tc::tc_fence_after();
      const long long q = T.q0 + r;
      const bool valid = q < g.NP;
      const int n = valid ? (int)(q / g.P) : 0;
      const int p = valid ? (int)(q - (long long)n * g.P) : 0;
      const long long obase = ((long long)n * g.outC + (long long)T.gi * g.Og + T.o0) * g.P + p;
      const int bbase = T.gi * g.Og + T.o0;
      const uint32_t ta = tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)(acc * tn);
      auto store = [&](int o, float v) {  // + bias, into the output
        const float y = v + (g.use_bias ? ld_io<FMT>(bias, bbase + o) : 0.f);
        const long long at = obase + (long long)o * g.P;
        if constexpr (H16)
          static_cast<unsigned short*>(out)[at] = to_h16<FMT>(y);
        else
          static_cast<float*>(out)[at] = y;
      };
      if (w.slot < 0) {  // whole tile
        for (int cb = 0; cb < tn; cb += 8) {
          float vv[8];
          tc::tmem_ld8(ta + (uint32_t)cb, vv);
          tc::tmem_ld_wait();
          if (valid) {
#pragma unroll
            for (int j = 0; j < 8; ++j) store(cb + j, vv[j]);
          }
        }
        tc::tc_fence_before();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
        return true;
      }
      // a piece of a split tile: its partial into the slot (out channel
      // major, so a warp's 32 rows are one 128-byte line); fwd_tail_sum_kernel
      // adds the pieces after the launch
      float* mine = tp.part + (size_t)w.slot * tn * BM;
      for (int cb = 0; cb < tn; cb += 8) {
        float vv[8];
        tc::tmem_ld8(ta + (uint32_t)cb, vv);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j) mine[(cb + j) * BM + r] = vv[j];
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&acc_empty[acc]);
      return true;
    });
  }

  tc::tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, (uint32_t)tcols);
  }
}

// The split tiles' sums: element e of tail tile j (e = o * BM + r: out
// channel o of the tile, pixel row r) is the sum of the tile's pieces' slots
// in CTA order -- the first CTA's slot 0 when its range starts in this tile,
// else its slot 1, then slot 0 of each later CTA -- plus the bias.
template <int FMT>
__global__ void __launch_bounds__(256) fwd_tail_sum_kernel(Geom g, TailPlan tp, int steps,
                                                           int mtiles, int ntiles_n, int tn,
                                                           const void* __restrict__ bias,
                                                           void* __restrict__ out) {
  const long long e = blockIdx.x * 256LL + threadIdx.x;
  const long long per_tile = (long long)tn * BM;
  const int j = (int)(e / per_tile);
  const int rem = (int)(e - (long long)j * per_tile);
  const int o = rem / BM, r = rem - o * BM;
  const Tile T = tile_of(tp.whole + j, mtiles, ntiles_n, tn);
  const long long q = T.q0 + r;
  if (j >= (int)(tp.tail_steps / steps) || q >= g.NP) return;
  const long long x0 = (long long)j * steps;
  const int cfirst = tail_cta_of(tp, x0), clast = tail_cta_of(tp, x0 + steps - 1);
  const bool first_starts_here = (long long)cfirst * tp.tail_steps / tp.ctas == x0;
  float v = __ldcg(tp.part + (size_t)(2 * cfirst + (first_starts_here ? 0 : 1)) * per_tile + rem);
  for (int c = cfirst + 1; c <= clast; ++c) v += __ldcg(tp.part + (size_t)(2 * c) * per_tile + rem);
  const int n = (int)(q / g.P);
  const int p = (int)(q - (long long)n * g.P);
  const int oc = T.gi * g.Og + T.o0 + o;
  const long long at = ((long long)n * g.outC + oc) * g.P + p;
  const float y = v + (g.use_bias ? ld_io<FMT>(bias, oc) : 0.f);
  if constexpr (FMT == kFmtF32) static_cast<float*>(out)[at] = y;
  else static_cast<unsigned short*>(out)[at] = to_h16<FMT>(y);
}

// Packed B operand: wt[(g*Og + o) * Kpad + k*Cg + c] = tf32(W[g*Og+o][c][k]);
// with `split`, rows outC .. 2*outC-1 hold the low parts tf32(W - hi).  One
// block per out channel: the (Cg x kk) row is read through L1 and written
// tap-major with coalesced stores.
__device__ __forceinline__ void pack_weight_row(long long oc, const float* __restrict__ w,
                                                float* __restrict__ wt, const Geom& g,
                                                int split) {
  const int Kpad = g.kk * g.Cg;
  const float* src = w + oc * Kpad;
  float* dst = wt + oc * Kpad;
  const long long lo = (long long)g.outC * Kpad;
  for (int j = threadIdx.x; j < Kpad; j += blockDim.x) {
    const int k = j / g.Cg, c = j - k * g.Cg;
    const float v = __ldg(src + c * g.kk + k);
    const float hi = tc::to_tf32(v);
    dst[j] = hi;
    if (split) dst[lo + j] = tc::to_tf32(v - hi);
  }
}
__global__ void __launch_bounds__(256) tc_pack_weight_kernel(const float* __restrict__ w,
                                                             float* __restrict__ wt, Geom g,
                                                             int split) {
  pack_weight_row(blockIdx.x, w, wt, g, split);
}

// The tensor-core forward's two helpers in one launch on the caller's
// stream: blocks [0, tiles) stage the NCHW input as its NHWC copy xt (64 x 64
// tiles; block 0 also zeroes the pixel row after it, the sampling plans'
// stand-in for out-of-image corners), the outC blocks after them pack the
// weight (tc_pack_weight_kernel's rows).  One launch instead of a transpose
// beside a side-stream pack saves the fork, the join and a launch gap in
// front of the forward kernel.
__global__ void __launch_bounds__(256) fwd_prologue_kernel(const float* __restrict__ x,
                                                           float* __restrict__ xt, int tiles_x,
                                                           int per_img, int tiles,
                                                           const float* __restrict__ w,
                                                           float* __restrict__ wt, Geom g,
                                                           int split) {
  __shared__ float tile[64][65];
  const int b = blockIdx.x;
  if (b < tiles) {
    const int n = b / per_img, r = b - n * per_img;
    transpose4_tile(x, xt, g.C, g.HW, n, r % tiles_x, r / tiles_x, tile, nullptr);
    if (b == 0) {
      float* zrow = xt + (long long)g.N * g.HW * g.C;
      for (int i = threadIdx.x; i < g.C; i += blockDim.x) zrow[i] = 0.f;
    }
  } else {
    pack_weight_row(b - tiles, w, wt, g, split);
  }
}

// 16-bit packed B operand: wt[(g*Og + o) * Kpad + k*Cg + c] = W[g*Og+o][c][k]
// (bf16 or fp16 words moved as they are, no rounding).
__global__ void __launch_bounds__(256) tc_pack_weight_bf16_kernel(
    const unsigned short* __restrict__ w, unsigned short* __restrict__ wt, Geom g) {
  const int Kpad = g.kk * g.Cg;
  const long long oc = blockIdx.x;
  const unsigned short* src = w + oc * Kpad;
  unsigned short* dst = wt + oc * Kpad;
  for (int j = threadIdx.x; j < Kpad; j += blockDim.x) {
    const int k = j / g.Cg, c = j - k * g.Cg;
    dst[j] = __ldg(src + c * g.kk + k);
  }
}

// 512 out channels a tile when the group has a multiple of 512 (not in
// 3xTF32, whose two operand parts would not fit two stages)
bool wide_tiles(int mode, const Geom& g) { return mode != kSplit && g.Og % 512 == 0; }
int tile_cols(int mode, const Geom& g) { return (wide_tiles(mode, g) ? 2 : 1) * tc_bn(g); }
long long tile_count(int mode, const Geom& g) {
  return (g.NP + BM - 1) / BM * (g.Og / tile_cols(mode, g)) * g.G;
}
int kstep_count(int mode, const Geom& g) {
  return g.kk * g.Cg / (mode == kBF16 || mode == kF16 ? 64 : 32);
}

// The schedule (TailPlan) of `ntiles` tiles of `steps` K steps on `num_sms`
// SMs: the last round is split when at least half the SMs would sit idle in
// it, the tiles have enough K steps to share (8 or more) and the cut leaves
// every CTA a quarter of a tile or more.  (The gather is bound by L2 -> SM
// throughput more than by each SM's latency: a last round on part of the SMs
// runs faster per tile than a full one, and the pieces' partial sums cost L2
// traffic, so a split pays only when most of the SMs would idle -- measured:
// 48 of 148 busy, forward -6%; 90 of 148, +3%; 108 of 148, +8%.)
struct TailShape {
  int grid = 0, whole = 0, ctas = 0;
  long long tail_steps = 0;
  size_t bytes = 0;  // scratch: 2 partial-sum slots a CTA
};
TailShape plan_tail(long long ntiles, int steps, int tn, int num_sms) {
  TailShape p;
  p.grid = (int)(ntiles < num_sms ? ntiles : num_sms);
  p.whole = (int)ntiles;
  if (steps < 8 || num_sms <= 0 || ntiles <= 0) return p;
  const long long whole = ntiles / num_sms * num_sms, tail = ntiles - whole;
  if (tail == 0 || tail > num_sms / 2) return p;
  const long long T = tail * steps;
  if (T >= (1LL << 30)) return p;
  const long long min_seg = steps / 4 > 2 ? steps / 4 : 2;
  long long ctas = T / min_seg < num_sms ? T / min_seg : num_sms;
  if (ctas <= tail) return p;                  // no more CTAs than tiles: nothing gained
  if ((T + ctas - 1) / ctas > steps) return p;  // ranges of at most one tile
  p.whole = (int)whole;
  p.ctas = (int)ctas;
  p.tail_steps = T;
  p.grid = whole > 0 ? num_sms : (int)ctas;
  p.bytes = (size_t)2 * ctas * tn * BM * sizeof(float);
  return p;
}

cudaError_t launch_fwd_mode(int mode, const Geom& g, const void* xt, const CUtensorMap& wmap,
                            const void* off, const void* mask, const void* bias, void* out,
                            void* tail, size_t tail_bytes, int num_sms, cudaStream_t stream) {
  const int bn = tc_bn(g);
  const bool wide = wide_tiles(mode, g);
  const int tn = tile_cols(mode, g);
  const size_t smem = wide ? 2 * ((size_t)A_STAGE + (size_t)tn * 128) + kBarrierBytes + 1024
                           : smem_bytes(bn, mode == kSplit);
  auto kern = mode == kSplit ? fwd_tc_kernel<kSplit, 1>
              : mode == kBF16 ? (wide ? fwd_tc_kernel<kBF16, 2> : fwd_tc_kernel<kBF16, 1>)
              : mode == kF16  ? (wide ? fwd_tc_kernel<kF16, 2> : fwd_tc_kernel<kF16, 1>)
                              : (wide ? fwd_tc_kernel<kTF32, 2> : fwd_tc_kernel<kTF32, 1>);
  cudaError_t e = ensure_dynamic_smem(reinterpret_cast<const void*>(kern), (int)smem);
  if (e != cudaSuccess) return e;
  const int mtiles = (int)((g.NP + BM - 1) / BM);
  const int ntiles_n = g.Og / tn;
  const long long ntiles = tile_count(mode, g);
  if (ntiles > (1LL << 30)) return cudaErrorInvalidValue;
  TailShape ts = plan_tail(ntiles, kstep_count(mode, g), tn, num_sms);
  if (ts.ctas > 0 && (tail == nullptr || tail_bytes < ts.bytes))  // no scratch: whole tiles
    ts = plan_tail(ntiles, 0, tn, num_sms);
  TailPlan tp;
  tp.whole = ts.whole;
  tp.ctas = ts.ctas;
  tp.tail_steps = ts.tail_steps;
  tp.part = ts.ctas > 0 ? static_cast<float*>(tail) : nullptr;
  kern<<<ts.grid, THREADS, smem, stream>>>(g, wmap, xt, bn, wide ? 512 : tmem_cols_for(bn),
                                            mtiles, ntiles_n, tp, off, mask, bias, out);
  e = cudaGetLastError();
  if (e != cudaSuccess || ts.ctas == 0) return e;
  // the split tiles' pieces, added in CTA order, + bias, into the output
  const long long elems = (ntiles - ts.whole) * (long long)tn * BM;
  const long long blocks = (elems + 255) / 256;
  if (blocks > (1LL << 31) - 1) return cudaErrorInvalidValue;
  const int steps = kstep_count(mode, g);
  auto sum = mode == kBF16 ? fwd_tail_sum_kernel<kFmtBF16>
             : mode == kF16 ? fwd_tail_sum_kernel<kFmtF16>
                            : fwd_tail_sum_kernel<kFmtF32>;
  sum<<<(unsigned)blocks, 256, 0, stream>>>(g, tp, steps, mtiles, ntiles_n, tn, bias, out);
  return cudaGetLastError();
}

}  // namespace

bool tc_fwd_supported(const Geom& g) {
  return g.Cg % 32 == 0 && g.cpg % 32 == 0 && g.C % 4 == 0 && g.Og % 16 == 0 &&
         (g.Og <= 256 || g.Og % 256 == 0) && g.NP > 0 &&
         (long long)g.N * g.HW * g.C + g.C < (1LL << 31) && (long long)g.kk * g.Cg < (1LL << 30);
}

size_t tc_fwd_weight_bytes(const Geom& g, bool split) {
  return (size_t)(split ? 2 : 1) * g.outC * g.kk * g.Cg * sizeof(float);
}

cudaError_t read_fwd_status(int* status, bool clear, cudaStream_t stream) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, g_tc_fwd_status, sizeof(int), 0,
                                            cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess && clear && v != 0) {
    const int zero = 0;
    e = cudaMemcpyToSymbolAsync(g_tc_fwd_status, &zero, sizeof(int), 0, cudaMemcpyHostToDevice,
                                stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  }
  *status = v;
  return e;
}

size_t tc_fwd_tail_bytes(const Geom& g, bool split, bool h16, int num_sms) {
  if (g.NP <= 0 || g.G <= 0) return 0;
  const int mode = split ? kSplit : (h16 ? kBF16 : kTF32);
  return plan_tail(tile_count(mode, g), kstep_count(mode, g), tile_cols(mode, g), num_sms).bytes;
}

bool fwd_prologue_fits(const float* x, const float* xt, const Geom& g) {
  return transpose4_fits(x, xt, g.C, g.HW) &&
         transpose4_tiles(g.N, g.C, g.HW) + g.outC <= (1LL << 31) - 1;
}

cudaError_t launch_fwd_prologue(const float* x, float* xt, const float* w, float* wt,
                                const Geom& g, bool split, cudaStream_t stream) {
  if (!fwd_prologue_fits(x, xt, g)) return cudaErrorInvalidValue;
  // x (N, C, HW) -> xt (N, HW, C): rows C, columns HW
  const int tiles_x = transpose4_tiles_x(g.HW);
  const int per_img = tiles_x * ((g.C + 63) / 64);
  const long long tiles = transpose4_tiles(g.N, g.C, g.HW);
  const long long blocks = tiles + ((long long)g.outC * g.kk * g.Cg > 0 ? g.outC : 0);
  if (blocks == 0) {  // nothing to stage or pack: the zero row alone
    return g.C > 0 ? cudaMemsetAsync(xt + (long long)g.N * g.HW * g.C, 0,
                                     (size_t)g.C * sizeof(float), stream)
                   : cudaSuccess;
  }
  if (tiles == 0) {  // an empty input: the zero row, then the pack
    cudaError_t e = g.C > 0 ? cudaMemsetAsync(xt, 0, (size_t)g.C * sizeof(float), stream)
                            : cudaSuccess;
    if (e != cudaSuccess) return e;
  }
  fwd_prologue_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, xt, tiles_x, per_img, (int)tiles,
                                                           w, wt, g, split ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_tc_pack_weight(const float* w, float* wt, const Geom& g, bool split,
                                  cudaStream_t stream) {
  if ((long long)g.outC * g.kk * g.Cg == 0) return cudaSuccess;
  tc_pack_weight_kernel<<<g.outC, 256, 0, stream>>>(w, wt, g, split ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_fwd_tc(const Geom& g, const float* xt, const float* wt, const float* off,
                          const float* mask, const float* bias, float* out, bool split,
                          void* tail, size_t tail_bytes, int num_sms, cudaStream_t stream) {
  if (!tc_fwd_supported(g)) return cudaErrorInvalidValue;
  const int Kpad = g.kk * g.Cg;
  CUtensorMap wmap;
  cudaError_t e = make_tmap_2d_f32(&wmap, wt, (uint64_t)Kpad,
                                   (uint64_t)g.outC * (split ? 2 : 1), (uint64_t)Kpad,
                                   (uint32_t)tc_bn(g));
  if (e != cudaSuccess) return e;
  return launch_fwd_mode(split ? kSplit : kTF32, g, xt, wmap, off, mask, bias, out, tail,
                         tail_bytes, num_sms,
                         stream);
}

bool tc_fwd_bf16_supported(const Geom& g) {
  return g.Cg % 64 == 0 && g.cpg % 64 == 0 && g.C % 8 == 0 && g.Og % 16 == 0 &&
         (g.Og <= 256 || g.Og % 256 == 0) && g.NP > 0 &&
         (long long)g.N * g.HW * g.C + g.C < (1LL << 31) && (long long)g.kk * g.Cg < (1LL << 30);
}

size_t tc_fwd_weight_bf16_bytes(const Geom& g) { return (size_t)g.outC * g.kk * g.Cg * 2; }

cudaError_t launch_tc_pack_weight_bf16(const void* w, void* wt, const Geom& g,
                                       cudaStream_t stream) {
  if ((long long)g.outC * g.kk * g.Cg == 0) return cudaSuccess;
  tc_pack_weight_bf16_kernel<<<g.outC, 256, 0, stream>>>(
      static_cast<const unsigned short*>(w), static_cast<unsigned short*>(wt), g);
  return cudaGetLastError();
}

cudaError_t launch_fwd_tc_bf16(const Geom& g, const void* xt, const void* wt, const void* off,
                               const void* mask, const void* bias, void* out, bool f16,
                               void* tail, size_t tail_bytes, int num_sms,
                               cudaStream_t stream) {
  if (!tc_fwd_bf16_supported(g)) return cudaErrorInvalidValue;
  const int Kpad = g.kk * g.Cg;
  CUtensorMap wmap;
  cudaError_t e = make_tmap_2d_bf16(&wmap, wt, (uint64_t)Kpad, (uint64_t)g.outC,
                                    (uint64_t)Kpad, (uint32_t)tc_bn(g), f16);
  if (e != cudaSuccess) return e;
  return launch_fwd_mode(f16 ? kF16 : kBF16, g, xt, wmap, off, mask, bias, out, tail, tail_bytes,
                         num_sms, stream);
}

}  // namespace dcn
