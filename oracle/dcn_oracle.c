/*
 * dcn_oracle.c -- CPU restatement of the reference deformable-convolution
 * algorithm.  TEST INFRASTRUCTURE ONLY: this file is the oracle that the
 * CUDA kernels are compared against.  It is never linked into, loaded by or
 * called from the product library; only tests/, the smoke entry and the
 * bench's CPU-baseline leg load it.
 *
 * What it restates (file:line within ilirium/pytorch_mps_deform_conv2d):
 *   bilinear_interpolate        src/deform_conv2d_mps/_C/bilinear.metalh:13-38
 *   get_gradient_weight         src/deform_conv2d_mps/_C/bilinear.metalh:46-69
 *   get_coordinate_weight       src/deform_conv2d_mps/_C/bilinear.metalh:73-99
 *   deformable_im2col           src/deform_conv2d_mps/_C/deform_conv2d.metal:74-125
 *   deformable_col2im           src/deform_conv2d_mps/_C/deform_conv2d.metal:141-204
 *   deformable_col2im_coord     src/deform_conv2d_mps/_C/deform_conv2d.metal:225-295
 *   deform_conv2d_forward host  src/deform_conv2d_mps/_C/deform_conv2d_mps.mm:192-374
 *   deform_conv2d_backward host src/deform_conv2d_mps/_C/deform_conv2d_mps.mm:682-890
 * Those kernels in turn restate torchvision's deform_conv2d (the reference's
 * CPU route, src/deform_conv2d_mps/ops.py:165-169); the boundary rules
 * (whole-sample cut at <= -1 / >= size, per-corner guards, the -2 sentinel
 * of the coordinate kernel, the mask gradient taken once per (tap, pixel))
 * are kept exactly.
 *
 * Arithmetic: the per-sample bilinear math is fp32 like the reference; every
 * reduction (the three GEMMs, the channel loop of the coordinate kernel, the
 * scatter-add of col2im and the bias sum) accumulates in double, so the
 * oracle is at least as accurate as the fp32 reference it restates.
 *
 * Layouts are the reference's: NCHW input, offset (N, 2*dg*kh*kw, Ho, Wo)
 * with (h, w) interleaved per tap, mask (N, dg*kh*kw, Ho, Wo), weight
 * (outC, C/groups, kh, kw), columns (C*kh*kw, Ho*Wo) with row c*kh*kw + k.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int64_t N, C, H, W, outC, kh, kw;
    int64_t sh, sw, ph, pw, dh, dw, groups, dg;
    int64_t Ho, Wo;
} geom_t;

static int make_geom(geom_t* g, int64_t N, int64_t C, int64_t H, int64_t W,
                     int64_t outC, int64_t kh, int64_t kw, int64_t sh,
                     int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                     int64_t dw, int64_t groups, int64_t dg) {
    g->N = N; g->C = C; g->H = H; g->W = W; g->outC = outC;
    g->kh = kh; g->kw = kw; g->sh = sh; g->sw = sw; g->ph = ph; g->pw = pw;
    g->dh = dh; g->dw = dw; g->groups = groups; g->dg = dg;
    /* output size: deform_conv2d_mps.mm:231-234 */
    g->Ho = (H + 2 * ph - dh * (kh - 1) - 1) / sh + 1;
    g->Wo = (W + 2 * pw - dw * (kw - 1) - 1) / sw + 1;
    if (groups <= 0 || dg <= 0 || C % groups || outC % groups || C % dg)
        return -1;
    return 0;
}

/* bilinear.metalh:13-38 */
static float bilinear(const float* in, int64_t height, int64_t width,
                      float h, float w) {
    if (h <= -1 || height <= h || w <= -1 || width <= w) return 0.0f;
    int64_t h_low = (int64_t)floorf(h), w_low = (int64_t)floorf(w);
    int64_t h_high = h_low + 1, w_high = w_low + 1;
    float lh = h - (float)h_low, lw = w - (float)w_low;
    float hh = 1.0f - lh, hw = 1.0f - lw;
    float v1 = (h_low >= 0 && w_low >= 0) ? in[h_low * width + w_low] : 0.0f;
    float v2 = (h_low >= 0 && w_high <= width - 1) ? in[h_low * width + w_high] : 0.0f;
    float v3 = (h_high <= height - 1 && w_low >= 0) ? in[h_high * width + w_low] : 0.0f;
    float v4 = (h_high <= height - 1 && w_high <= width - 1) ? in[h_high * width + w_high] : 0.0f;
    float w1 = hh * hw, w2 = hh * lw, w3 = lh * hw, w4 = lh * lw;
    return w1 * v1 + w2 * v2 + w3 * v3 + w4 * v4;
}

/* bilinear.metalh:46-69 */
static float gradient_weight(float ah, float aw, int64_t h, int64_t w,
                             int64_t height, int64_t width) {
    if (ah <= -1 || ah >= height || aw <= -1 || aw >= width) return 0.0f;
    int64_t h_low = (int64_t)floorf(ah), w_low = (int64_t)floorf(aw);
    int64_t h_high = h_low + 1, w_high = w_low + 1;
    float weight = 0.0f;
    if (h == h_low && w == w_low) weight = ((float)h + 1 - ah) * ((float)w + 1 - aw);
    if (h == h_low && w == w_high) weight = ((float)h + 1 - ah) * (aw + 1 - (float)w);
    if (h == h_high && w == w_low) weight = (ah + 1 - (float)h) * ((float)w + 1 - aw);
    if (h == h_high && w == w_high) weight = (ah + 1 - (float)h) * (aw + 1 - (float)w);
    return weight;
}

/* bilinear.metalh:73-99 */
static float coordinate_weight(const float* in, int64_t height, int64_t width,
                               float h, float w, int bp_dir) {
    if (h <= -1 || height <= h || w <= -1 || width <= w) return 0.0f;
    int64_t h_low = (int64_t)floorf(h), w_low = (int64_t)floorf(w);
    int64_t h_high = h_low + 1, w_high = w_low + 1;
    float lh = h - (float)h_low, lw = w - (float)w_low;
    float v1 = (h_low >= 0 && w_low >= 0) ? in[h_low * width + w_low] : 0.0f;
    float v2 = (h_low >= 0 && w_high <= width - 1) ? in[h_low * width + w_high] : 0.0f;
    float v3 = (h_high <= height - 1 && w_low >= 0) ? in[h_high * width + w_low] : 0.0f;
    float v4 = (h_high <= height - 1 && w_high <= width - 1) ? in[h_high * width + w_high] : 0.0f;
    if (bp_dir == 0) return (1.0f - lw) * (v3 - v1) + lw * (v4 - v2);
    return (1.0f - lh) * (v2 - v1) + lh * (v4 - v3);
}

/* deform_conv2d.metal:74-125 -- one image; col is (C*kk, Ho*Wo). */
static void im2col(const geom_t* g, const float* im, const float* off,
                   const float* msk, float* col) {
    const int64_t kk = g->kh * g->kw, hw = g->Ho * g->Wo;
    const int64_t cpg = g->C / g->dg;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < g->C; ++c) {
        const int64_t dgi = c / cpg;
        const float* plane = im + c * g->H * g->W;
        for (int64_t oy = 0; oy < g->Ho; ++oy)
            for (int64_t ox = 0; ox < g->Wo; ++ox)
                for (int64_t ki = 0; ki < g->kh; ++ki)
                    for (int64_t kj = 0; kj < g->kw; ++kj) {
                        const int64_t k = ki * g->kw + kj;
                        const int64_t oh_idx = ((2 * (dgi * kk + k)) * g->Ho + oy) * g->Wo + ox;
                        const int64_t ow_idx = ((2 * (dgi * kk + k) + 1) * g->Ho + oy) * g->Wo + ox;
                        const float h_im = (float)(oy * g->sh - g->ph + ki * g->dh) + off[oh_idx];
                        const float w_im = (float)(ox * g->sw - g->pw + kj * g->dw) + off[ow_idx];
                        float val = bilinear(plane, g->H, g->W, h_im, w_im);
                        if (msk) val *= msk[((dgi * kk + k) * g->Ho + oy) * g->Wo + ox];
                        col[(c * kk + k) * hw + oy * g->Wo + ox] = val;
                    }
    }
}

/* deform_conv2d.metal:141-204 -- one image; scatters col into grad_im
 * (C, H, W), which the caller zeroes.  The reference's +-2 window with the
 * |delta| < 1 guard visits exactly the in-bounds corners of the sample, so
 * the scan below keeps that window and that guard. */
static void col2im(const geom_t* g, const float* col, const float* off,
                   const float* msk, double* grad_im) {
    const int64_t kk = g->kh * g->kw, hw = g->Ho * g->Wo;
    const int64_t cpg = g->C / g->dg;
#pragma omp parallel for schedule(static)
    for (int64_t c = 0; c < g->C; ++c) {  /* channel-parallel: no races */
        const int64_t dgi = c / cpg;
        double* plane = grad_im + c * g->H * g->W;
        for (int64_t k = 0; k < kk; ++k) {
            const int64_t ki = k / g->kw, kj = k % g->kw;
            for (int64_t oy = 0; oy < g->Ho; ++oy)
                for (int64_t ox = 0; ox < g->Wo; ++ox) {
                    const int64_t oh_idx = ((2 * (dgi * kk + k)) * g->Ho + oy) * g->Wo + ox;
                    const int64_t ow_idx = ((2 * (dgi * kk + k) + 1) * g->Ho + oy) * g->Wo + ox;
                    const float h_im = (float)(oy * g->sh - g->ph + ki * g->dh) + off[oh_idx];
                    const float w_im = (float)(ox * g->sw - g->pw + kj * g->dw) + off[ow_idx];
                    float top = col[(c * kk + k) * hw + oy * g->Wo + ox];
                    if (msk) top *= msk[((dgi * kk + k) * g->Ho + oy) * g->Wo + ox];
                    const int64_t cur_h = (int64_t)floorf(h_im), cur_w = (int64_t)floorf(w_im);
                    for (int64_t dy = -2; dy <= 2; ++dy)
                        for (int64_t dx = -2; dx <= 2; ++dx) {
                            const int64_t yp = cur_h + dy, xp = cur_w + dx;
                            if (yp >= 0 && yp < g->H && xp >= 0 && xp < g->W &&
                                fabsf(h_im - (float)yp) < 1.0f &&
                                fabsf(w_im - (float)xp) < 1.0f) {
                                const float wt = gradient_weight(h_im, w_im, yp, xp, g->H, g->W);
                                plane[yp * g->W + xp] += (double)(wt * top);
                            }
                        }
                }
        }
    }
}

/* deform_conv2d.metal:225-295 -- one image. */
static void col2im_coord(const geom_t* g, const float* col, const float* im,
                         const float* off, const float* msk, float* grad_off,
                         float* grad_msk) {
    const int64_t kk = g->kh * g->kw, hw = g->Ho * g->Wo;
    const int64_t cpg = g->C / g->dg;
    const int64_t total = 2 * g->dg * kk * hw;
#pragma omp parallel for schedule(static)
    for (int64_t gid = 0; gid < total; ++gid) {
        const int64_t ox = gid % g->Wo, oy = (gid / g->Wo) % g->Ho, c = gid / hw;
        const int64_t dgi = c / (2 * kk), offset_c = c - dgi * 2 * kk;
        const int bp_dir = (int)(offset_c % 2);
        const int64_t k = offset_c / 2, ki = k / g->kw, kj = k % g->kw;
        const int64_t oh_idx = ((2 * (dgi * kk + k)) * g->Ho + oy) * g->Wo + ox;
        const int64_t ow_idx = ((2 * (dgi * kk + k) + 1) * g->Ho + oy) * g->Wo + ox;
        const int64_t m_idx = ((dgi * kk + k) * g->Ho + oy) * g->Wo + ox;
        const float mask_value = msk ? msk[m_idx] : 1.0f;
        float inv_h = (float)(oy * g->sh - g->ph + ki * g->dh) + off[oh_idx];
        float inv_w = (float)(ox * g->sw - g->pw + kj * g->dw) + off[ow_idx];
        if (inv_h <= -1 || inv_w <= -1 || inv_h >= g->H || inv_w >= g->W)
            inv_h = inv_w = -2.0f;  /* sentinel: deform_conv2d.metal:268-270 */
        double val = 0.0, mval = 0.0;
        for (int64_t ch = 0; ch < cpg; ++ch) {
            const int64_t c_im = dgi * cpg + ch;
            const float* plane = im + c_im * g->H * g->W;
            const float col_v = col[(c_im * kk + k) * hw + oy * g->Wo + ox];
            const float wt = coordinate_weight(plane, g->H, g->W, inv_h, inv_w, bp_dir);
            val += (double)mask_value * (double)wt * (double)col_v;
            if (msk && bp_dir == 0)
                mval += (double)col_v * (double)bilinear(plane, g->H, g->W, inv_h, inv_w);
        }
        grad_off[gid] = (float)val;
        if (msk && bp_dir == 0) grad_msk[m_idx] = (float)mval;
    }
}

/* ------------------------------------------------------------------------ */
/* Exported entry points (ctypes).  All pointers are host fp32 buffers.      */
/* ------------------------------------------------------------------------ */

int oracle_geom_out(int64_t H, int64_t W, int64_t kh, int64_t kw, int64_t sh,
                    int64_t sw, int64_t ph, int64_t pw, int64_t dh,
                    int64_t dw, int64_t* Ho, int64_t* Wo) {
    *Ho = (H + 2 * ph - dh * (kh - 1) - 1) / sh + 1;
    *Wo = (W + 2 * pw - dw * (kw - 1) - 1) / sw + 1;
    return (*Ho > 0 && *Wo > 0) ? 0 : -1;
}

/* deform_conv2d_mps.mm:192-374: per image im2col, grouped GEMM, bias. */
int oracle_forward(const float* x, const float* w, const float* off,
                   const float* msk, const float* bias, float* out,
                   int64_t N, int64_t C, int64_t H, int64_t W, int64_t outC,
                   int64_t kh, int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                   int64_t pw, int64_t dh, int64_t dw, int64_t groups,
                   int64_t dg) {
    geom_t g;
    if (make_geom(&g, N, C, H, W, outC, kh, kw, sh, sw, ph, pw, dh, dw, groups, dg)) return -1;
    const int64_t kk = kh * kw, hw = g.Ho * g.Wo;
    const int64_t Cg = C / groups, Og = outC / groups, Kg = Cg * kk;
    float* col = (float*)malloc(sizeof(float) * (size_t)(C * kk * hw + 1));
    if (!col) return -2;
    for (int64_t n = 0; n < N; ++n) {
        im2col(&g, x + n * C * H * W, off + n * 2 * dg * kk * hw,
               msk ? msk + n * dg * kk * hw : NULL, col);
        float* o_n = out + n * outC * hw;
#pragma omp parallel for schedule(static)
        for (int64_t o = 0; o < outC; ++o) {
            const int64_t gi = o / Og;
            const float* wrow = w + o * Kg;           /* (Cg, kh, kw) == Kg */
            const float* cg = col + gi * Kg * hw;     /* rows gi*Kg .. */
            double* acc = (double*)calloc((size_t)hw, sizeof(double));
            for (int64_t r = 0; r < Kg; ++r) {
                const double wv = wrow[r];
                const float* crow = cg + r * hw;
                for (int64_t p = 0; p < hw; ++p) acc[p] += wv * crow[p];
            }
            const double b = bias ? bias[o] : 0.0;
            for (int64_t p = 0; p < hw; ++p) o_n[o * hw + p] = (float)(acc[p] + b);
            free(acc);
        }
    }
    free(col);
    return 0;
}

/* deform_conv2d_mps.mm:682-890: per image grad_col = W^T go, coordinate
 * kernel, col2im, im2col recompute, grad_weight += go col^T; grad_bias =
 * go.sum(0, 2, 3).  grad_mask / grad_bias may be NULL (DCNv1 / no bias). */
int oracle_backward(const float* go, const float* x, const float* w,
                    const float* off, const float* msk, float* gx,
                    float* goff, float* gmsk, float* gw, float* gb,
                    int64_t N, int64_t C, int64_t H, int64_t W, int64_t outC,
                    int64_t kh, int64_t kw, int64_t sh, int64_t sw,
                    int64_t ph, int64_t pw, int64_t dh, int64_t dw,
                    int64_t groups, int64_t dg) {
    geom_t g;
    if (make_geom(&g, N, C, H, W, outC, kh, kw, sh, sw, ph, pw, dh, dw, groups, dg)) return -1;
    const int64_t kk = kh * kw, hw = g.Ho * g.Wo;
    const int64_t Cg = C / groups, Og = outC / groups, Kg = Cg * kk;
    float* gcol = (float*)malloc(sizeof(float) * (size_t)(C * kk * hw + 1));
    float* col = (float*)malloc(sizeof(float) * (size_t)(C * kk * hw + 1));
    double* gim = (double*)malloc(sizeof(double) * (size_t)(C * H * W + 1));
    double* gwacc = (double*)calloc((size_t)(outC * Kg + 1), sizeof(double));
    if (!gcol || !col || !gim || !gwacc) { free(gcol); free(col); free(gim); free(gwacc); return -2; }
    for (int64_t n = 0; n < N; ++n) {
        const float* go_n = go + n * outC * hw;
        const float* x_n = x + n * C * H * W;
        const float* off_n = off + n * 2 * dg * kk * hw;
        const float* msk_n = msk ? msk + n * dg * kk * hw : NULL;
        /* 1. grad_columns = W_g^T @ go_g   (.mm:820-821) */
#pragma omp parallel for schedule(static)
        for (int64_t rr = 0; rr < C * kk; ++rr) {
            const int64_t gi = rr / Kg, r = rr % Kg;
            double* acc = (double*)calloc((size_t)hw, sizeof(double));
            for (int64_t o = 0; o < Og; ++o) {
                const double wv = w[(gi * Og + o) * Kg + r];
                const float* grow = go_n + (gi * Og + o) * hw;
                for (int64_t p = 0; p < hw; ++p) acc[p] += wv * grow[p];
            }
            for (int64_t p = 0; p < hw; ++p) gcol[rr * hw + p] = (float)acc[p];
            free(acc);
        }
        /* 2. coordinate kernel -> grad_offset[n], grad_mask[n] (.mm:824-831) */
        col2im_coord(&g, gcol, x_n, off_n, msk_n, goff + n * 2 * dg * kk * hw,
                     msk_n ? gmsk + n * dg * kk * hw : NULL);
        /* 3. col2im -> grad_input[n] (.mm:834-837) */
        memset(gim, 0, sizeof(double) * (size_t)(C * H * W));
        col2im(&g, gcol, off_n, msk_n, gim);
        for (int64_t i = 0; i < C * H * W; ++i) gx[n * C * H * W + i] = (float)gim[i];
        /* 4. recompute columns (.mm:842-875) */
        im2col(&g, x_n, off_n, msk_n, col);
        /* 5. grad_weight += go_g @ col_g^T (.mm:880) */
#pragma omp parallel for schedule(static)
        for (int64_t o = 0; o < outC; ++o) {
            const int64_t gi = o / Og;
            const float* grow = go_n + o * hw;
            for (int64_t r = 0; r < Kg; ++r) {
                const float* crow = col + (gi * Kg + r) * hw;
                double s = 0.0;
                for (int64_t p = 0; p < hw; ++p) s += (double)grow[p] * crow[p];
                gwacc[o * Kg + r] += s;
            }
        }
    }
    for (int64_t i = 0; i < outC * Kg; ++i) gw[i] = (float)gwacc[i];
    if (gb) { /* .mm:885-886 */
        for (int64_t o = 0; o < outC; ++o) {
            double s = 0.0;
            for (int64_t n = 0; n < N; ++n)
                for (int64_t p = 0; p < hw; ++p) s += go[(n * outC + o) * hw + p];
            gb[o] = (float)s;
        }
    }
    free(gcol); free(col); free(gim); free(gwacc);
    return 0;
}

/* Single-image building blocks with the reference's debug-op contracts
 * (deform_conv2d_mps.mm:388-504 and :516-651). */
int oracle_col2im(const float* col, const float* off, const float* msk,
                  float* grad_im, int64_t C, int64_t H, int64_t W, int64_t kh,
                  int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                  int64_t dh, int64_t dw, int64_t dg) {
    geom_t g;
    if (make_geom(&g, 1, C, H, W, C, kh, kw, sh, sw, ph, pw, dh, dw, 1, dg)) return -1;
    double* gim = (double*)calloc((size_t)(C * H * W + 1), sizeof(double));
    if (!gim) return -2;
    col2im(&g, col, off, msk, gim);
    for (int64_t i = 0; i < C * H * W; ++i) grad_im[i] = (float)gim[i];
    free(gim);
    return 0;
}

int oracle_col2im_coord(const float* col, const float* im, const float* off,
                        const float* msk, float* grad_off, float* grad_msk,
                        int64_t C, int64_t H, int64_t W, int64_t kh,
                        int64_t kw, int64_t sh, int64_t sw, int64_t ph,
                        int64_t pw, int64_t dh, int64_t dw, int64_t dg) {
    geom_t g;
    if (make_geom(&g, 1, C, H, W, C, kh, kw, sh, sw, ph, pw, dh, dw, 1, dg)) return -1;
    col2im_coord(&g, col, im, off, msk, grad_off, grad_msk);
    return 0;
}

/* Raw column buffer for one image (used by the unfold-parity ladder). */
int oracle_im2col(const float* im, const float* off, const float* msk,
                  float* col, int64_t C, int64_t H, int64_t W, int64_t kh,
                  int64_t kw, int64_t sh, int64_t sw, int64_t ph, int64_t pw,
                  int64_t dh, int64_t dw, int64_t dg) {
    geom_t g;
    if (make_geom(&g, 1, C, H, W, C, kh, kw, sh, sw, ph, pw, dh, dw, 1, dg)) return -1;
    im2col(&g, im, off, msk, col);
    return 0;
}
