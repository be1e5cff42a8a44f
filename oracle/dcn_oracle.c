/*
 * dcn_oracle.c -- CPU restatement of the deformable-convolution path of
 * mps-deform-conv, in double precision.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity oracle: the tests, the
 * smoke check and the bench's CPU-baseline leg may call it as the checker.
 * The product (the CUDA kernels behind include/dcn_b200.h) never links,
 * loads or calls it.
 *
 * Pinned against torchvision.ops.deform_conv2d (CPU, float64) by the committed
 * fixtures in tests/golden/ (made by tests/golden/make_golden.py): forward and
 * all five gradients, groups, offset groups, stride, dilation, masks and
 * out-of-bounds samples.
 *
 * Tensor layouts are the reference's (all row-major, NCHW):
 *   input   [B][C][H][W]
 *   offset  [B][og][kh][kw][2][Ho][Wo]   (dy at even, dx at odd channel)
 *   mask    [B][og][kh][kw][Ho][Wo]
 *   weight  [Co][C/g][kh][kw]
 *   columns [C*kh*kw][B*Ho*Wo]           (row = c*kh*kw + tap)
 *   output  [B][Co][Ho][Wo]
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

typedef struct {
    int64_t B, C, H, W;     /* input */
    int64_t Co, kh, kw;     /* weight */
    int64_t sh, sw, ph, pw, dh, dw;
    int64_t groups, og;     /* weight groups, offset groups */
    int64_t use_mask;
    int64_t Ho, Wo;         /* derived */
} dcn_oracle_shape;

static void fill_out_size(dcn_oracle_shape *s) {
    /* mps_deform_conv/__init__.py:208-209 */
    s->Ho = (s->H + 2 * s->ph - (s->dh * (s->kh - 1) + 1)) / s->sh + 1;
    s->Wo = (s->W + 2 * s->pw - (s->dw * (s->kw - 1) + 1)) / s->sw + 1;
}

/* Bilinear sample of one HxW plane; zero outside (-1, H) x (-1, W) and per
 * corner.  Follows csrc/deform_conv2d_mps.mm:41-68. */
static double bilinear(const double *plane, int64_t H, int64_t W, double y, double x) {
    if (y <= -1.0 || (double)H <= y || x <= -1.0 || (double)W <= x) return 0.0;
    int64_t y0 = (int64_t)floor(y), x0 = (int64_t)floor(x);
    int64_t y1 = y0 + 1, x1 = x0 + 1;
    double ly = y - (double)y0, lx = x - (double)x0;
    double hy = 1.0 - ly, hx = 1.0 - lx;
    double v00 = (y0 >= 0 && x0 >= 0) ? plane[y0 * W + x0] : 0.0;
    double v01 = (y0 >= 0 && x1 <= W - 1) ? plane[y0 * W + x1] : 0.0;
    double v10 = (y1 <= H - 1 && x0 >= 0) ? plane[y1 * W + x0] : 0.0;
    double v11 = (y1 <= H - 1 && x1 <= W - 1) ? plane[y1 * W + x1] : 0.0;
    return hy * hx * v00 + hy * lx * v01 + ly * hx * v10 + ly * lx * v11;
}

/* d(bilinear)/dy (is_y) or d/dx, with per-corner validity and no global
 * out-of-range exit.  Follows csrc/deform_conv2d_mps.mm:72-102. */
static double coord_weight(const double *plane, int64_t H, int64_t W, double y, double x, int is_y) {
    int64_t y0 = (int64_t)floor(y), x0 = (int64_t)floor(x);
    int64_t y1 = y0 + 1, x1 = x0 + 1;
    int vy0 = 0 <= y0 && y0 < H, vy1 = 0 <= y1 && y1 < H;
    int vx0 = 0 <= x0 && x0 < W, vx1 = 0 <= x1 && x1 < W;
    double v00 = (vy0 && vx0) ? plane[y0 * W + x0] : 0.0;
    double v01 = (vy0 && vx1) ? plane[y0 * W + x1] : 0.0;
    double v10 = (vy1 && vx0) ? plane[y1 * W + x0] : 0.0;
    double v11 = (vy1 && vx1) ? plane[y1 * W + x1] : 0.0;
    if (is_y) {
        double fx = x - (double)x0;
        return fx * (v11 - v01) + (1.0 - fx) * (v10 - v00);
    } else {
        double fy = y - (double)y0;
        return fy * (v11 - v10) + (1.0 - fy) * (v01 - v00);
    }
}

/* Sampling position of tap t at output pixel (oy, ox) for (b, g_off).
 * Follows csrc/deform_conv2d_mps.mm:154-168. */
static void sample_pos(const dcn_oracle_shape *s, const double *offset, int64_t b, int64_t go,
                       int64_t t, int64_t oy, int64_t ox, double *y, double *x) {
    int64_t T = s->kh * s->kw, HWo = s->Ho * s->Wo;
    int64_t i = t / s->kw, j = t % s->kw;
    const double *op = offset + ((b * s->og + go) * 2 * T) * HWo;
    double dy = op[(2 * t) * HWo + oy * s->Wo + ox];
    double dx = op[(2 * t + 1) * HWo + oy * s->Wo + ox];
    *y = (double)(oy * s->sh - s->ph) + (double)(i * s->dh) + dy;
    *x = (double)(ox * s->sw - s->pw) + (double)(j * s->dw) + dx;
}

static double mask_at(const dcn_oracle_shape *s, const double *mask, int64_t b, int64_t go,
                      int64_t t, int64_t oy, int64_t ox) {
    if (!s->use_mask) return 1.0;
    int64_t T = s->kh * s->kw, HWo = s->Ho * s->Wo;
    return mask[((b * s->og + go) * T + t) * HWo + oy * s->Wo + ox];
}

/* columns[c*T + t][b*HWo + p] = mask * bilinear(input[b, c], y, x).
 * Follows deformable_im2col_fp32, csrc/deform_conv2d_mps.mm:105-174. */
void dcn_oracle_im2col(const dcn_oracle_shape *sin, const double *input, const double *offset,
                       const double *mask, double *columns) {
    dcn_oracle_shape s = *sin;
    fill_out_size(&s);
    int64_t T = s.kh * s.kw, HWo = s.Ho * s.Wo, P = s.B * HWo;
    int64_t cpg = s.C / s.og;
    for (int64_t c = 0; c < s.C; ++c) {
        int64_t go = c / cpg;
        for (int64_t b = 0; b < s.B; ++b) {
            const double *plane = input + (b * s.C + c) * s.H * s.W;
            for (int64_t t = 0; t < T; ++t) {
                double *col = columns + (c * T + t) * P + b * HWo;
                for (int64_t oy = 0; oy < s.Ho; ++oy)
                    for (int64_t ox = 0; ox < s.Wo; ++ox) {
                        double y, x;
                        sample_pos(&s, offset, b, go, t, oy, ox, &y, &x);
                        col[oy * s.Wo + ox] =
                            mask_at(&s, mask, b, go, t, oy, ox) * bilinear(plane, s.H, s.W, y, x);
                    }
            }
        }
    }
}

/* grad_input += col2im(grad_columns): the transpose of the bilinear gather,
 * weight (1-|y-yp|)(1-|x-xp|) on the 3x3 window around trunc(y), trunc(x).
 * Follows deformable_col2im_fp32, csrc/deform_conv2d_mps.mm:344-417.
 * grad_input must be zeroed by the caller. */
void dcn_oracle_col2im(const dcn_oracle_shape *sin, const double *grad_columns, const double *offset,
                       const double *mask, double *grad_input) {
    dcn_oracle_shape s = *sin;
    fill_out_size(&s);
    int64_t T = s.kh * s.kw, HWo = s.Ho * s.Wo, P = s.B * HWo;
    int64_t cpg = s.C / s.og;
    for (int64_t c = 0; c < s.C; ++c) {
        int64_t go = c / cpg;
        for (int64_t t = 0; t < T; ++t)
            for (int64_t b = 0; b < s.B; ++b) {
                double *gplane = grad_input + (b * s.C + c) * s.H * s.W;
                const double *gcol = grad_columns + (c * T + t) * P + b * HWo;
                for (int64_t oy = 0; oy < s.Ho; ++oy)
                    for (int64_t ox = 0; ox < s.Wo; ++ox) {
                        double y, x;
                        sample_pos(&s, offset, b, go, t, oy, ox, &y, &x);
                        double m = mask_at(&s, mask, b, go, t, oy, ox);
                        double v = gcol[oy * s.Wo + ox];
                        int64_t ty = (int64_t)y, tx = (int64_t)x; /* C truncation, as int(y) */
                        for (int64_t ddy = -1; ddy <= 1; ++ddy)
                            for (int64_t ddx = -1; ddx <= 1; ++ddx) {
                                int64_t yp = ty + ddy, xp = tx + ddx;
                                if (0 <= yp && yp < s.H && 0 <= xp && xp < s.W &&
                                    fabs(y - (double)yp) < 1.0 && fabs(x - (double)xp) < 1.0) {
                                    double wgt = (1.0 - fabs(y - (double)yp)) * (1.0 - fabs(x - (double)xp));
                                    gplane[yp * s.W + xp] += m * wgt * v;
                                }
                            }
                    }
            }
    }
}

/* grad_offset[b, og, t, {y,x}, p] = sum_c mask * coord_weight * gcol
 * grad_mask[b, og, t, p]           = sum_c gcol * bilinear
 * Follows deformable_col2im_coord_fp32, csrc/deform_conv2d_mps.mm:423-519.
 * Both outputs are fully overwritten; grad_mask may be NULL when !use_mask. */
void dcn_oracle_col2im_coord(const dcn_oracle_shape *sin, const double *grad_columns,
                             const double *input, const double *offset, const double *mask,
                             double *grad_offset, double *grad_mask) {
    dcn_oracle_shape s = *sin;
    fill_out_size(&s);
    int64_t T = s.kh * s.kw, HWo = s.Ho * s.Wo, P = s.B * HWo;
    int64_t cpg = s.C / s.og;
    for (int64_t b = 0; b < s.B; ++b)
        for (int64_t go = 0; go < s.og; ++go)
            for (int64_t t = 0; t < T; ++t)
                for (int64_t oy = 0; oy < s.Ho; ++oy)
                    for (int64_t ox = 0; ox < s.Wo; ++ox) {
                        double y, x;
                        sample_pos(&s, offset, b, go, t, oy, ox, &y, &x);
                        double m = mask_at(&s, mask, b, go, t, oy, ox);
                        double gy = 0.0, gx = 0.0, gm = 0.0;
                        for (int64_t cl = 0; cl < cpg; ++cl) {
                            int64_t c = go * cpg + cl;
                            const double *plane = input + (b * s.C + c) * s.H * s.W;
                            double v = grad_columns[(c * T + t) * P + b * HWo + oy * s.Wo + ox];
                            gy += m * coord_weight(plane, s.H, s.W, y, x, 1) * v;
                            gx += m * coord_weight(plane, s.H, s.W, y, x, 0) * v;
                            if (s.use_mask) gm += v * bilinear(plane, s.H, s.W, y, x);
                        }
                        int64_t obase = ((b * s.og + go) * 2 * T) * HWo + oy * s.Wo + ox;
                        grad_offset[obase + (2 * t) * HWo] = gy;
                        grad_offset[obase + (2 * t + 1) * HWo] = gx;
                        if (s.use_mask && grad_mask)
                            grad_mask[((b * s.og + go) * T + t) * HWo + oy * s.Wo + ox] = gm;
                    }
}

/* Full forward: im2col, then per weight group out = W_g . cols_g (+ bias),
 * stored NCHW.  Follows csrc/deform_conv2d_mps.mm:603-800 (grouped bmm at
 * :765-782, permute and bias at :785-792).  bias may be NULL. */
void dcn_oracle_forward(const dcn_oracle_shape *sin, const double *input, const double *offset,
                        const double *mask, const double *weight, const double *bias, double *output) {
    dcn_oracle_shape s = *sin;
    fill_out_size(&s);
    int64_t T = s.kh * s.kw, HWo = s.Ho * s.Wo, P = s.B * HWo;
    int64_t Cig = s.C / s.groups, Cog = s.Co / s.groups, K = Cig * T;
    double *cols = (double *)malloc(sizeof(double) * (size_t)(s.C * T * (P > 0 ? P : 1)));
    dcn_oracle_im2col(&s, input, offset, mask, cols);
    double *acc = (double *)malloc(sizeof(double) * (size_t)(P > 0 ? P : 1));
    for (int64_t g = 0; g < s.groups; ++g)
        for (int64_t co = 0; co < Cog; ++co) {
            int64_t oc = g * Cog + co;
            for (int64_t p = 0; p < P; ++p) acc[p] = 0.0;
            for (int64_t k = 0; k < K; ++k) {
                double w = weight[oc * K + k];
                const double *crow = cols + (g * K + k) * P;
                for (int64_t p = 0; p < P; ++p) acc[p] += w * crow[p];
            }
            double bv = bias ? bias[oc] : 0.0;
            for (int64_t b = 0; b < s.B; ++b)
                for (int64_t p = 0; p < HWo; ++p)
                    output[(b * s.Co + oc) * HWo + p] = acc[b * HWo + p] + bv;
        }
    free(acc);
    free(cols);
}

/* Full backward with per-group GEMMs.  The reference's autograd backward
 * (mps_deform_conv/__init__.py:245-322) flattens the weight across groups at
 * :281 and :289-290, which is only valid for groups == 1; this restatement
 * uses the per-group products that the forward's grouped bmm implies.
 * Any output pointer may be NULL to skip it.  grad_mask is only written when
 * use_mask. */
void dcn_oracle_backward(const dcn_oracle_shape *sin, const double *grad_out, const double *input,
                         const double *offset, const double *mask, const double *weight,
                         double *grad_input, double *grad_offset, double *grad_mask,
                         double *grad_weight, double *grad_bias) {
    dcn_oracle_shape s = *sin;
    fill_out_size(&s);
    int64_t T = s.kh * s.kw, HWo = s.Ho * s.Wo, P = s.B * HWo;
    int64_t Cig = s.C / s.groups, Cog = s.Co / s.groups, K = Cig * T;
    size_t colsz = (size_t)(s.C * T * (P > 0 ? P : 1));
    /* grad_out as [Co][P] (__init__.py:276) */
    double *go = (double *)malloc(sizeof(double) * (size_t)(s.Co * (P > 0 ? P : 1)));
    for (int64_t b = 0; b < s.B; ++b)
        for (int64_t oc = 0; oc < s.Co; ++oc)
            memcpy(go + oc * P + b * HWo, grad_out + (b * s.Co + oc) * HWo, sizeof(double) * (size_t)HWo);
    if (grad_bias) /* __init__.py:286 */
        for (int64_t oc = 0; oc < s.Co; ++oc) {
            double a = 0.0;
            for (int64_t p = 0; p < P; ++p) a += go[oc * P + p];
            grad_bias[oc] = a;
        }
    if (grad_weight) { /* __init__.py:266-281, per group */
        double *cols = (double *)malloc(sizeof(double) * colsz);
        dcn_oracle_im2col(&s, input, offset, mask, cols);
        for (int64_t g = 0; g < s.groups; ++g)
            for (int64_t co = 0; co < Cog; ++co)
                for (int64_t k = 0; k < K; ++k) {
                    const double *grow = go + (g * Cog + co) * P;
                    const double *crow = cols + (g * K + k) * P;
                    double a = 0.0;
                    for (int64_t p = 0; p < P; ++p) a += grow[p] * crow[p];
                    grad_weight[(g * Cog + co) * K + k] = a;
                }
        free(cols);
    }
    if (grad_input || grad_offset || grad_mask) { /* __init__.py:289-316, per group */
        double *gcol = (double *)calloc(colsz, sizeof(double));
        for (int64_t g = 0; g < s.groups; ++g)
            for (int64_t co = 0; co < Cog; ++co) {
                const double *grow = go + (g * Cog + co) * P;
                for (int64_t k = 0; k < K; ++k) {
                    double w = weight[(g * Cog + co) * K + k];
                    double *gc = gcol + (g * K + k) * P;
                    for (int64_t p = 0; p < P; ++p) gc[p] += w * grow[p];
                }
            }
        if (grad_input) {
            memset(grad_input, 0, sizeof(double) * (size_t)(s.B * s.C * s.H * s.W));
            dcn_oracle_col2im(&s, gcol, offset, mask, grad_input);
        }
        if (grad_offset || grad_mask) {
            double *goff = grad_offset ? grad_offset
                                       : (double *)malloc(sizeof(double) * (size_t)(s.B * s.og * 2 * T * (HWo > 0 ? HWo : 1)));
            dcn_oracle_col2im_coord(&s, gcol, input, offset, mask, goff, grad_mask);
            if (!grad_offset) free(goff);
        }
        free(gcol);
    }
    free(go);
}

void dcn_oracle_out_size(const dcn_oracle_shape *sin, int64_t *Ho, int64_t *Wo) {
    dcn_oracle_shape s = *sin;
    fill_out_size(&s);
    *Ho = s.Ho;
    *Wo = s.Wo;
}
