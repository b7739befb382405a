// dcn_fwd_tc.cu -- forward deformable convolution on the 5th-generation
// tensor cores (tcgen05, kind::tf32, fp32 accumulation in tensor memory).
//
// Implicit GEMM per group g:  D[pixels, out channels] = A . B^T with
//   A[q, (k, c)] = mask * bilinear(x[n, c], sample(q, k))   (deform_conv2d.metal:74-125)
//   B[o, (k, c)] = W[g*Og + o, c, k]
// K ordered (tap, channel); a K step is 32 channels of one tap (128 bytes of
// tf32 per row, one 128-byte swizzle atom row).  The column matrix A never
// touches HBM: 8 warps gather it per K step straight into swizzled shared
// memory (4 corners per sample, 16-byte loads of the NHWC input; 16 loads in
// flight per thread), while the weight tile arrives by cp.async.  One thread
// issues four 128xBNx8 UMMAs per K step into a tensor-memory accumulator;
// their completion (tcgen05.commit -> mbarrier) releases the stage.  Two
// stages per CTA, two CTAs per SM, so one CTA's gather overlaps the other's
// MMAs and epilogue.  Epilogue: tcgen05.ld -> +bias -> NCHW stores.
//
// Operands are rounded to TF32 with round-to-nearest (cvt.rna) when they are
// staged, so the products carry an unbiased 2^-11 relative error instead of
// the truncation bias of feeding raw fp32.
#include "dcn_tc.h"
#include "dcn_tc_common.cuh"

namespace dcn {

__device__ int g_tc_fwd_status;  // set to 1 by a wait that ran out

namespace {

constexpr int BM = 128;
constexpr int THREADS = 256;
constexpr int ROUNDS = 4;  // rows per lane: 8 warps x 4 rounds x 4 sub-rows = 128

int tc_bn(const Geom& g) { return g.Og <= 256 ? g.Og : 256; }
int tmem_cols(int bn) {
  int c = 32;
  while (c < bn) c <<= 1;
  return c;
}
size_t smem_bytes(int bn) { return 2 * 16384 + 2 * (size_t)bn * 128 + 64 + 1024; }

__global__ void __launch_bounds__(THREADS, 2)
fwd_tc_kernel(Geom g, const float* __restrict__ xt, const float* __restrict__ wt, int Kpad,
              int bn, int tcols, const float* __restrict__ off, const float* __restrict__ mask,
              const float* __restrict__ bias, float* __restrict__ out) {
  extern __shared__ unsigned char smem_raw[];
  const uint32_t raw_u32 = tc::smem_u32(smem_raw);
  unsigned char* smem = smem_raw + ((1024u - (raw_u32 & 1023u)) & 1023u);
  const uint32_t sA0 = tc::smem_u32(smem);
  const uint32_t sB0 = sA0 + 2 * 16384;
  const uint32_t b_stage = (uint32_t)bn * 128;
  uint64_t* mma_bar = reinterpret_cast<uint64_t*>(smem + 2 * 16384 + 2 * b_stage);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_bar + 2);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const long long q0 = (long long)blockIdx.x * BM;
  const int o0 = blockIdx.y * bn;
  const int gi = blockIdx.z;
  const int nchunk = g.Cg >> 5;
  const int steps = g.kk * nchunk;

  if (tid == 0) {
    tc::mbar_init(&mma_bar[0], 1);
    tc::mbar_init(&mma_bar[1], 1);
    tc::fence_mbar_init();
  }
  if (warp == 0) {
    tc::tmem_alloc(tmem_slot, (uint32_t)tcols);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // ---- gather role: rows warp*16 + i*4 + sub, channel quad `quad` ----
  const int quad = lane & 7, sub = lane >> 3;
  int rn[ROUNDS], rp[ROUNDS], roy[ROUNDS], rox[ROUNDS];
  bool rvalid[ROUNDS];
#pragma unroll
  for (int i = 0; i < ROUNDS; ++i) {
    const long long q = q0 + warp * 16 + i * 4 + sub;
    rvalid[i] = q < g.NP;
    const int n = rvalid[i] ? (int)(q / g.P) : 0;
    const int p = rvalid[i] ? (int)(q - (long long)n * g.P) : 0;
    rn[i] = n;
    rp[i] = p;
    roy[i] = p / g.Wo;
    rox[i] = p - roy[i] * g.Wo;
  }
  int cidx[ROUNDS][4];
  float cw[ROUNDS][4];
  int cached_k = -1, cached_dgi = -1;
  const uint32_t idesc = tc::idesc_tf32(BM, bn);
  const float* wsrc = wt + (size_t)(gi * g.Og + o0) * Kpad;

  for (int s = 0; s < steps; ++s) {
    const int st = s & 1;
    const int k = s / nchunk;
    const int c0 = (s - k * nchunk) << 5;
    const int gch0 = gi * g.Cg + c0;
    const int dgi = gch0 / g.cpg;
    if (s >= 2) tc::mbar_wait(&mma_bar[st], ((s - 2) >> 1) & 1, &g_tc_fwd_status);

    // weight tile: bn rows x 128 B, cp.async into the swizzled stage
    const uint32_t sB = sB0 + st * b_stage;
    for (int i = tid; i < bn * 8; i += THREADS) {
      const int o = i >> 3, j = i & 7;
      tc::cp_async16(sB + tc::sw128_offset(o, j), wsrc + (size_t)o * Kpad + s * 32 + j * 4);
    }

    // sampling plans of this lane's rows for (tap k, deformable group dgi)
    if (k != cached_k || dgi != cached_dgi) {
      cached_k = k;
      cached_dgi = dgi;
      const int ki = k / g.kw, kj = k - ki * g.kw;
#pragma unroll
      for (int i = 0; i < ROUNDS; ++i) {
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          cidx[i][c] = -1;
          cw[i][c] = 0.f;
        }
        if (!rvalid[i]) continue;
        const long long oi = off_h_index(g, rn[i], dgi, k, rp[i]);
        const float h = (float)(roy[i] * g.sh - g.ph + ki * g.dh) + __ldg(off + oi);
        const float w = (float)(rox[i] * g.sw - g.pw + kj * g.dw) + __ldg(off + oi + g.P);
        const float m = g.use_mask ? __ldg(mask + mask_index(g, rn[i], dgi, k, rp[i])) : 1.f;
        const Sample sp = make_sample(h, w, g.H, g.W);
        if (!sp.valid) continue;
        const int nb = rn[i] * g.HW;
        if (sp.live & 1u) { cidx[i][0] = nb + sp.i1; cw[i][0] = sp.w1 * m; }
        if (sp.live & 2u) { cidx[i][1] = nb + sp.i2; cw[i][1] = sp.w2 * m; }
        if (sp.live & 4u) { cidx[i][2] = nb + sp.i3; cw[i][2] = sp.w3 * m; }
        if (sp.live & 8u) { cidx[i][3] = nb + sp.i4; cw[i][3] = sp.w4 * m; }
      }
    }

    // gather: all 16 loads first, then combine
    float4 v[ROUNDS][4];
    const float* xq = xt + gch0 + quad * 4;
#pragma unroll
    for (int i = 0; i < ROUNDS; ++i)
#pragma unroll
      for (int c = 0; c < 4; ++c)
        v[i][c] = cidx[i][c] >= 0 ? ldg4(xq + (size_t)cidx[i][c] * g.C)
                                  : make_float4(0.f, 0.f, 0.f, 0.f);
    const uint32_t sA = sA0 + st * 16384;
#pragma unroll
    for (int i = 0; i < ROUNDS; ++i) {
      const float a = cw[i][0], b = cw[i][1], c = cw[i][2], d = cw[i][3];
      const float4 A = v[i][0], B = v[i][1], C = v[i][2], D = v[i][3];
      tc::st_shared_v4(sA + tc::sw128_offset(warp * 16 + i * 4 + sub, quad),
                       tc::to_tf32(a * A.x + b * B.x + c * C.x + d * D.x),
                       tc::to_tf32(a * A.y + b * B.y + c * C.y + d * D.y),
                       tc::to_tf32(a * A.z + b * B.z + c * C.z + d * D.z),
                       tc::to_tf32(a * A.w + b * B.w + c * C.w + d * D.w));
    }
    tc::cp_async_wait_all();
    tc::fence_proxy_async();
    __syncthreads();
    if (tid == 0) {
      tc::tc_fence_after();
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::umma_tf32(tmem, tc::sdesc_sw128(sA + j * 32), tc::sdesc_sw128(sB + j * 32), idesc,
                      (s | j) != 0 ? 1u : 0u);
      tc::umma_commit(&mma_bar[st]);
    }
  }

  // ---- epilogue: wait for the last commit, TMEM -> registers -> NCHW ----
  const int last = steps - 1;
  tc::mbar_wait(&mma_bar[last & 1], (last >> 1) & 1, &g_tc_fwd_status);
  tc::tc_fence_after();
  {
    const int lq = warp & 3, half = warp >> 2;
    const int r = lq * 32 + lane;
    const long long q = q0 + r;
    const bool valid = q < g.NP;
    const int n = valid ? (int)(q / g.P) : 0;
    const int p = valid ? (int)(q - (long long)n * g.P) : 0;
    float* orow = out + ((long long)n * g.outC + (long long)gi * g.Og + o0) * g.P + p;
    const int cbeg = half * (bn >> 1), cend = cbeg + (bn >> 1);
    for (int cb = cbeg; cb < cend; cb += 8) {
      float vv[8];
      tc::tmem_ld8(tmem + ((uint32_t)(lq * 32) << 16) + (uint32_t)cb, vv);
      tc::tmem_ld_wait();
      if (valid) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int o = cb + j;
          const float bv = g.use_bias ? __ldg(bias + gi * g.Og + o0 + o) : 0.f;
          orow[(long long)o * g.P] = vv[j] + bv;
        }
      }
    }
  }
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, (uint32_t)tcols);
  }
}

// Packed B operand: wt[(g*Og + o) * Kpad + k*Cg + c] = tf32(W[g*Og+o][c][k]).
__global__ void tc_pack_weight_kernel(const float* __restrict__ w, float* __restrict__ wt,
                                      Geom g) {
  const int Kpad = g.kk * g.Cg;
  const long long total = (long long)g.outC * Kpad;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
       i += (long long)gridDim.x * blockDim.x) {
    const int kc = (int)(i % Kpad);
    const long long oc = i / Kpad;
    const int k = kc / g.Cg, c = kc - k * g.Cg;
    wt[i] = tc::to_tf32(w[(oc * g.Cg + c) * g.kk + k]);
  }
}

}  // namespace

bool tc_fwd_supported(const Geom& g) {
  return g.Cg % 32 == 0 && g.cpg % 32 == 0 && g.C % 4 == 0 && g.Og % 16 == 0 &&
         (g.Og <= 256 || g.Og % 256 == 0) && g.NP > 0 &&
         (long long)g.N * g.HW < (1LL << 31) && g.kk * g.Cg < (1 << 30);
}

size_t tc_fwd_weight_bytes(const Geom& g) {
  return (size_t)g.outC * g.kk * g.Cg * sizeof(float);
}

cudaError_t launch_tc_pack_weight(const float* w, float* wt, const Geom& g, cudaStream_t stream) {
  const long long total = (long long)g.outC * g.kk * g.Cg;
  if (total == 0) return cudaSuccess;
  long long blocks = (total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  tc_pack_weight_kernel<<<(int)blocks, 256, 0, stream>>>(w, wt, g);
  return cudaGetLastError();
}

cudaError_t launch_fwd_tc(const Geom& g, const float* xt, const float* wt, const float* off,
                          const float* mask, const float* bias, float* out, int num_sms,
                          cudaStream_t stream) {
  (void)num_sms;
  if (!tc_fwd_supported(g)) return cudaErrorInvalidValue;
  const int bn = tc_bn(g);
  const size_t smem = smem_bytes(bn);
  cudaError_t e = cudaFuncSetAttribute(fwd_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid((unsigned)((g.NP + BM - 1) / BM), g.Og / bn, g.G);
  fwd_tc_kernel<<<grid, THREADS, smem, stream>>>(g, xt, wt, g.kk * g.Cg, bn, tmem_cols(bn), off,
                                                  mask, bias, out);
  return cudaGetLastError();
}

}  // namespace dcn
