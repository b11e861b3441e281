/*
 * gs_train_oracle.c -- CPU restatement of the reference's tiled training rasteriser and
 * its exact 2D backward, for parity checks at the benchmark configurations' full sizes.
 *
 * TEST INFRASTRUCTURE ONLY: the checker the CUDA training kernels are compared against;
 * libgs200.so never links or loads it.
 *
 * It restates, per tile and in the same fp32 operation order, the two numpy models of
 * oracle/train.py, which are themselves pinned to the reference's numpy models
 * (tests/test_oracle_train.py) and which this file reproduces bit for bit in the forward
 * and to the order of float64 additions in the backward (tests/test_oracle_train_c.py):
 *
 *   gso_train_forward   -- oracle/train.py forward, i.e. gsplat/blend_backward_dev.py:404-438
 *                          forward_fast: tile-centred power (gsplat/blend_backward_ref.py:68-92),
 *                          alpha = min(o * exp(min(power, 0)), alpha_max), skip below
 *                          alpha_min, stop before T would fall below t_min.
 *   gso_train_backward  -- oracle/train.py backward_2d_exact: the reference's per-pair
 *                          2D-gradient terms (gsplat/blend_backward_ref.py:134-249) on the
 *                          fp32 forward's decisions, accumulated back to front in float64 and
 *                          summed per Gaussian (gsplat/t2_param_backward.py:50-61).
 *
 * The numpy models sweep every pair of every tile; a tile here stops at the first pair
 * after which no pixel is alive (every later pair contributes nothing), except that the
 * tie marking of the backward keeps scanning while a pixel of the tile is tainted, as the
 * numpy model's marking does. Tiles are spread over POSIX threads; per-Gaussian sums use
 * atomic float64 additions (their order varies, ~1e-16 relative). exp is evaluated in
 * float64 and rounded once to float, as the numpy models do.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gs_oracle.h"

#define TIE_RTOL 4e-6f /* gsplat/blend_backward_dev.py:441 (about 32 fp32 ulp) */
#define MAX_TILE 32

typedef struct {
    const float *m2, *con, *op, *col;
    const int64_t *ids, *ranges;
    int H, W, tile, tx, ty;
    float amax, amin, tmin, bg[3];
    /* forward outputs */
    float *image, *final_T;
    int32_t *n_contrib;
    uint8_t *ties;
    int64_t *tile_reach;
    /* backward inputs / outputs */
    const float *dimg;
    double *grads;
    uint8_t *tie_g;
    int64_t next_tile;
    int64_t n_live;
} Job;

static int near_th(float q, float th) { return fabsf(q / th - 1.0f) < TIE_RTOL; }

/* exp rounded once to float from float64 (oracle/train.py _exp). */
static float exp1(float x) { return (float)exp((double)x); }

/* oracle/train.py _centred (gsplat/blend_backward_ref.py:68-85): coefficients of the
 * power about the tile centre, formed in float64 from the fp32 conic and rounded once. */
typedef struct { float Af, Bf, Cf, P0, Lx, Ly, mxl, myl; } Coef;

static Coef centred(const Job* J, int64_t g, float ox, float oy) {
    Coef c;
    const float A = J->con[3 * g], B = J->con[3 * g + 1], C = J->con[3 * g + 2];
    c.Af = -0.5f * A;
    c.Bf = -B;
    c.Cf = -0.5f * C;
    c.mxl = J->m2[2 * g] - ox;
    c.myl = J->m2[2 * g + 1] - oy;
    const double a = c.Af, b = c.Bf, cc = c.Cf;
    const double centre = (double)(float)(J->tile / 2.0);
    const double U0 = centre - (double)c.mxl, V0 = centre - (double)c.myl;
    const double P0 = a * U0 * U0 + b * U0 * V0 + cc * V0 * V0;
    const double Lx = 2.0 * a * U0 + b * V0;
    const double Ly = b * U0 + 2.0 * cc * V0;
    c.P0 = (float)P0;
    c.Lx = (float)Lx;
    c.Ly = (float)Ly;
    return c;
}

/* The fp32 power at pixel offset (du, dv) from the tile centre, in the numpy model's
 * order: P0 + du * (Lx + Af du + Bf dv) + dv * (Ly + Cf dv). */
static float power_at(const Coef* c, float du, float dv) {
    const float t4 = (c->Lx + c->Af * du) + c->Bf * dv;
    const float t6 = c->P0 + du * t4;
    const float t8 = c->Ly + c->Cf * dv;
    return t6 + dv * t8;
}

static void atomic_add_f64(double* p, double v) {
    uint64_t* u = (uint64_t*)p;
    uint64_t old = __atomic_load_n(u, __ATOMIC_RELAXED);
    for (;;) {
        double cur;
        memcpy(&cur, &old, 8);
        const double nv = cur + v;
        uint64_t nu;
        memcpy(&nu, &nv, 8);
        if (__atomic_compare_exchange_n(u, &old, nu, 1, __ATOMIC_RELAXED, __ATOMIC_RELAXED)) return;
    }
}

typedef struct {
    float T[MAX_TILE * MAX_TILE];
    float C[MAX_TILE * MAX_TILE][3];
    int32_t ks[MAX_TILE * MAX_TILE];  /* first pair index the pixel does not blend past */
    uint8_t inside[MAX_TILE * MAX_TILE], done[MAX_TILE * MAX_TILE], taint[MAX_TILE * MAX_TILE];
    int32_t ncon[MAX_TILE * MAX_TILE];
    float du[MAX_TILE], xx[MAX_TILE];
} TileState;

/* The fp32 forward of one tile (decisions of both numpy models). Returns the number of
 * leading pairs after which no pixel is alive; fills T, C, ncon, ks, taint. */
static int64_t tile_forward(const Job* J, int64_t t, TileState* S, int64_t* live_count) {
    const int tile = J->tile, np = tile * tile;
    const int64_t beg = J->ranges[2 * t], end = J->ranges[2 * t + 1];
    const float ox = (float)((t % J->tx) * tile), oy = (float)((t / J->tx) * tile);
    const float centre = (float)(tile / 2.0);
    for (int i = 0; i < tile; ++i) {
        S->xx[i] = (float)i + 0.5f;
        S->du[i] = S->xx[i] - centre;
    }
    int alive = 0;
    for (int p = 0; p < np; ++p) {
        const int px = (int)ox + p % tile, py = (int)oy + p / tile;
        S->inside[p] = px < J->W && py < J->H;
        S->done[p] = !S->inside[p];
        S->taint[p] = 0;
        S->T[p] = 1.0f;
        S->C[p][0] = S->C[p][1] = S->C[p][2] = 0.0f;
        S->ncon[p] = 0;
        S->ks[p] = (int32_t)(end - beg);
        alive += S->inside[p];
    }
    int64_t k = 0;
    int64_t nl = 0;
    for (; k < end - beg && alive > 0; ++k) {
        const int64_t g = J->ids[beg + k];
        const Coef c = centred(J, g, ox, oy);
        const float o = J->op[g];
        const float* col = J->col + 3 * g;
        for (int p = 0; p < np; ++p) {
            if (S->done[p]) continue;
            const float pw = power_at(&c, S->du[p % tile], S->du[p / tile]);
            const float raw = o * exp1(pw < 0.0f ? pw : 0.0f);
            const float al = raw < J->amax ? raw : J->amax;
            const float Tn = S->T[p] * (1.0f - al);
            if (near_th(al, J->amin) || near_th(raw, J->amax) || (al >= J->amin && near_th(Tn, J->tmin)))
                S->taint[p] = 1;
            if (!(al >= J->amin)) continue;
            if (Tn >= J->tmin) {
                const float w = al * S->T[p];
                for (int ch = 0; ch < 3; ++ch) S->C[p][ch] = S->C[p][ch] + w * col[ch];
                S->T[p] = Tn;
                S->ncon[p] = (int32_t)(k + 1);
                ++nl;
            } else {
                S->done[p] = 1;
                S->ks[p] = (int32_t)k;
                --alive;
            }
        }
    }
    *live_count += nl;
    return k;
}

static void* forward_worker(void* arg) {
    Job* J = (Job*)arg;
    TileState* S = (TileState*)malloc(sizeof(TileState));
    int64_t nl = 0;
    const int64_t ntiles = (int64_t)J->tx * J->ty;
    for (;;) {
        const int64_t t = __atomic_fetch_add(&J->next_tile, 1, __ATOMIC_RELAXED);
        if (t >= ntiles) break;
        const int64_t reach = tile_forward(J, t, S, &nl);
        if (J->tile_reach) J->tile_reach[t] = reach;
        const int tile = J->tile;
        const int ox = (int)(t % J->tx) * tile, oy = (int)(t / J->tx) * tile;
        for (int p = 0; p < tile * tile; ++p) {
            if (!S->inside[p]) continue;
            const int64_t pix = (int64_t)(oy + p / tile) * J->W + (ox + p % tile);
            for (int ch = 0; ch < 3; ++ch)
                J->image[3 * pix + ch] = S->C[p][ch] + S->T[p] * J->bg[ch];
            J->final_T[pix] = S->T[p];
            J->n_contrib[pix] = S->ncon[p];
            J->ties[pix] = S->taint[p];
        }
    }
    __atomic_fetch_add(&J->n_live, nl, __ATOMIC_RELAXED);
    free(S);
    return NULL;
}

static void* backward_worker(void* arg) {
    Job* J = (Job*)arg;
    TileState* S = (TileState*)malloc(sizeof(TileState));
    double* Gp = (double*)malloc(sizeof(double) * 3 * MAX_TILE * MAX_TILE);
    double* Tc = (double*)malloc(sizeof(double) * MAX_TILE * MAX_TILE);
    double* behind = (double*)malloc(sizeof(double) * MAX_TILE * MAX_TILE);
    int64_t nl = 0;
    const int64_t ntiles = (int64_t)J->tx * J->ty;
    const int tile = J->tile, np = tile * tile;
    const float amin_tie = J->amin * (1.0f - TIE_RTOL);
    for (;;) {
        const int64_t t = __atomic_fetch_add(&J->next_tile, 1, __ATOMIC_RELAXED);
        if (t >= ntiles) break;
        const int64_t beg = J->ranges[2 * t], end = J->ranges[2 * t + 1];
        if (end <= beg) continue;
        const int64_t kn = tile_forward(J, t, S, &nl);
        const float ox = (float)((t % J->tx) * tile), oy = (float)((t / J->tx) * tile);
        /* tie marking: every pair with alpha >= amin (1 - rtol) at a pixel tainted at or
         * before it (oracle/train.py backward_2d_exact, ties=True) */
        if (J->tie_g) {
            /* replay the taint in order: a pixel's taint at pair k counts from k on */
            uint8_t tnow[MAX_TILE * MAX_TILE];
            uint8_t alive[MAX_TILE * MAX_TILE];
            float T[MAX_TILE * MAX_TILE];
            int any_taint_final = 0;
            for (int p = 0; p < np; ++p) {
                tnow[p] = 0;
                alive[p] = S->inside[p];
                T[p] = 1.0f;
                any_taint_final |= S->taint[p];
            }
            const int64_t kscan = any_taint_final ? end - beg : kn;
            for (int64_t k = 0; k < kscan; ++k) {
                const int64_t g = J->ids[beg + k];
                const Coef c = centred(J, g, ox, oy);
                const float o = J->op[g];
                int mark = 0;
                for (int p = 0; p < np; ++p) {
                    if (!alive[p] && !tnow[p]) continue;
                    const float pw = power_at(&c, S->du[p % tile], S->du[p / tile]);
                    const float raw = o * exp1(pw < 0.0f ? pw : 0.0f);
                    const float al = raw < J->amax ? raw : J->amax;
                    if (alive[p]) {
                        const int live = al >= J->amin;
                        const float Tn = T[p] * (1.0f - al);
                        if (near_th(al, J->amin) || near_th(raw, J->amax) || (live && near_th(Tn, J->tmin)))
                            tnow[p] = 1;
                        if (live) {
                            if (Tn < J->tmin) alive[p] = 0;
                            else T[p] = Tn;
                        }
                    }
                    if (tnow[p] && al >= amin_tie) mark = 1;
                }
                if (mark) J->tie_g[g] = 1;
            }
        }
        /* back to front in float64 over the pairs [0, kn) */
        for (int p = 0; p < np; ++p) {
            const int px = (int)ox + p % tile, py = (int)oy + p / tile;
            double gb = 0.0;
            for (int ch = 0; ch < 3; ++ch) {
                const double v = S->inside[p] ? (double)J->dimg[3 * ((int64_t)py * J->W + px) + ch] : 0.0;
                Gp[3 * p + ch] = v;
                gb += v * (double)J->bg[ch];
            }
            Tc[p] = (double)S->T[p];
            behind[p] = Tc[p] * gb;
        }
        for (int64_t k = kn - 1; k >= 0; --k) {
            const int64_t g = J->ids[beg + k];
            const Coef c = centred(J, g, ox, oy);
            const float o = J->op[g];
            const float* col = J->col + 3 * g;
            double s[9] = {0, 0, 0, 0, 0, 0, 0, 0, 0};
            for (int p = 0; p < np; ++p) {
                if (!S->inside[p] || k >= S->ks[p]) continue;  /* dead or stopped here */
                const float pw = power_at(&c, S->du[p % tile], S->du[p / tile]);
                const float wgt = exp1(pw < 0.0f ? pw : 0.0f);
                const float raw = o * wgt;
                const int clamp = raw > J->amax;
                const float alpha = clamp ? J->amax : raw;
                if (!(alpha >= J->amin)) continue;           /* skipped: no terms */
                const double a = alpha, w = wgt;
                const double cg = (double)col[0] * Gp[3 * p] + (double)col[1] * Gp[3 * p + 1] +
                                  (double)col[2] * Gp[3 * p + 2];
                const double Ti = Tc[p] / (1.0 - a);
                const double dal = Ti * cg - behind[p] / (1.0 - a);
                const double at = a * Ti;
                behind[p] += at * cg;
                Tc[p] = Ti;
                const double u = (double)(S->xx[p % tile] - c.mxl);
                const double v = (double)(S->xx[p / tile] - c.myl);
                const double G = (!clamp && pw <= 0.0f) ? dal * a : 0.0;
                if (!clamp) s[0] += dal * w;
                s[1] += at * Gp[3 * p];
                s[2] += at * Gp[3 * p + 1];
                s[3] += at * Gp[3 * p + 2];
                s[4] += G * u * u;
                s[5] += G * u * v;
                s[6] += G * v * v;
                s[7] += G * u;
                s[8] += G * v;
            }
            const double Ac = J->con[3 * g], Bc = J->con[3 * g + 1], Cc = J->con[3 * g + 2];
            const double pair[9] = {Ac * s[7] + Bc * s[8], Bc * s[7] + Cc * s[8], -0.5 * s[4],
                                    -s[5], -0.5 * s[6], s[0], s[1], s[2], s[3]};
            double* dst = J->grads + 9 * g;
            for (int i = 0; i < 9; ++i)
                if (pair[i] != 0.0) atomic_add_f64(dst + i, pair[i]);
        }
    }
    free(S);
    free(Gp);
    free(Tc);
    free(behind);
    return NULL;
}

static int run_threads(Job* J, void* (*fn)(void*), int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t th[256];
    int started = 0;
    for (int i = 1; i < threads; ++i) {
        if (pthread_create(&th[started], NULL, fn, J) != 0) break;
        ++started;
    }
    fn(J);
    for (int i = 0; i < started; ++i) pthread_join(th[i], NULL);
    return 0;
}

static int fill_job(Job* J, const float* means2d, const float* conic, const float* opacity,
                    const float* colors, const int64_t* sorted_ids, const int64_t* tile_ranges,
                    int height, int width, int tile, float alpha_max, float alpha_min,
                    float t_min, const float* background) {
    if (tile < 1 || tile > MAX_TILE) return -1;
    memset(J, 0, sizeof(*J));
    J->m2 = means2d;
    J->con = conic;
    J->op = opacity;
    J->col = colors;
    J->ids = sorted_ids;
    J->ranges = tile_ranges;
    J->H = height;
    J->W = width;
    J->tile = tile;
    J->tx = (width + tile - 1) / tile;
    J->ty = (height + tile - 1) / tile;
    J->amax = alpha_max;
    J->amin = alpha_min;
    J->tmin = t_min;
    for (int i = 0; i < 3; ++i) J->bg[i] = background ? background[i] : 0.0f;
    return 0;
}

int64_t gso_train_forward(const float* means2d, const float* conic, const float* opacity,
                          const float* colors, const int64_t* sorted_ids,
                          const int64_t* tile_ranges, int height, int width, int tile,
                          float alpha_max, float alpha_min, float t_min, const float* background,
                          float* image, float* final_T, int32_t* n_contrib, uint8_t* ties,
                          int64_t* tile_reach, int threads) {
    Job J;
    if (fill_job(&J, means2d, conic, opacity, colors, sorted_ids, tile_ranges, height, width,
                 tile, alpha_max, alpha_min, t_min, background) != 0)
        return -1;
    J.image = image;
    J.final_T = final_T;
    J.n_contrib = n_contrib;
    J.ties = ties;
    J.tile_reach = tile_reach;
    run_threads(&J, forward_worker, threads);
    return J.n_live;
}

int gso_train_backward(const float* means2d, const float* conic, const float* opacity,
                       const float* colors, const int64_t* sorted_ids,
                       const int64_t* tile_ranges, int height, int width, int tile,
                       float alpha_max, float alpha_min, float t_min, const float* background,
                       const float* dL_dimage, int64_t n, double* grads, uint8_t* tie_gaussians,
                       int threads) {
    Job J;
    if (fill_job(&J, means2d, conic, opacity, colors, sorted_ids, tile_ranges, height, width,
                 tile, alpha_max, alpha_min, t_min, background) != 0)
        return -1;
    J.dimg = dL_dimage;
    J.grads = grads;
    J.tie_g = tie_gaussians;
    memset(grads, 0, sizeof(double) * 9 * (size_t)n);
    if (tie_gaussians) memset(tie_gaussians, 0, (size_t)n);
    run_threads(&J, backward_worker, threads);
    return 0;
}
