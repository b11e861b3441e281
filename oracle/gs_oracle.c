/*
 * gs_oracle.c -- serial C restatement of the reference's display-path stages.
 *
 * TEST INFRASTRUCTURE ONLY (see gs_oracle.h). Built with -ffp-contract=off so every
 * float product and sum rounds separately, in the operation order the reference
 * writes (citations are to the reference project's src/gsplat_cpu/ files).
 */
#include "gs_oracle.h"

#include <limits.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

static inline float fmaxf_ref(float a, float b) { return (a < b) ? b : a; } /* std::max */
static inline float fminf_ref(float a, float b) { return (b < a) ? b : a; } /* std::min */
static inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* types.h:68-97 quat_to_rotation_matrix + build_covariance_3d. */
static void cov3d_one(const float* s, const float* q, float* out) {
    const float w = q[0], x = q[1], y = q[2], z = q[3];
    float r[9];
    r[0] = 1.0f - 2.0f * (y * y + z * z);
    r[1] = 2.0f * (x * y - w * z);
    r[2] = 2.0f * (x * z + w * y);
    r[3] = 2.0f * (x * y + w * z);
    r[4] = 1.0f - 2.0f * (x * x + z * z);
    r[5] = 2.0f * (y * z - w * x);
    r[6] = 2.0f * (x * z - w * y);
    r[7] = 2.0f * (y * z + w * x);
    r[8] = 1.0f - 2.0f * (x * x + y * y);
    for (int col = 0; col < 3; ++col)
        for (int row = 0; row < 3; ++row) r[row * 3 + col] *= s[col];
    for (int i = 0; i < 3; ++i)
        for (int j = 0; j < 3; ++j)
            out[i * 3 + j] = r[i * 3 + 0] * r[j * 3 + 0] + r[i * 3 + 1] * r[j * 3 + 1] +
                             r[i * 3 + 2] * r[j * 3 + 2];
}

void gso_compute_cov3d(const float* scales, const float* quats, int64_t n, float* cov3d) {
    for (int64_t i = 0; i < n; ++i) cov3d_one(scales + 3 * i, quats + 4 * i, cov3d + 9 * i);
}

/* types.h:141-144 opacity_aware_k (logf/sqrtf of the host C library). */
static float opacity_k(float op, float floor_) {
    const float arg = fmaxf_ref(op / floor_, 1.0f);
    return sqrtf(2.0f * logf(arg));
}

int64_t gso_project(const float* means, const float* cov3d, const float* e, const float* k,
                    const float* colors, const float* opacities, float min_opacity, int64_t n,
                    int height, int width, int max_radius_param, float contrib_floor_k,
                    float k_cap, float* means_2d, float* covs_2d, float* depths, float* radii,
                    uint8_t* valid_mask, float* colors_out, float* opacities_out) {
    /* project.cpp:502-513: rotation rows, translation column, intrinsics, radius cap. */
    const float r00 = e[0], r01 = e[1], r02 = e[2], t0 = e[3];
    const float r10 = e[4], r11 = e[5], r12 = e[6], t1 = e[7];
    const float r20 = e[8], r21 = e[9], r22 = e[10], t2 = e[11];
    const float fx = k[0], fy = k[4], cx = k[2], cy = k[5];
    const int max_radius = max_radius_param < 0
                               ? INT_MAX
                               : (max_radius_param > 0 ? max_radius_param
                                                       : (height < width ? height : width) / 2);
    const float max_r = (float)max_radius;
    int64_t m = 0;
    for (int64_t i = 0; i < n; ++i) {
        const float mx = means[3 * i], my = means[3 * i + 1], mz = means[3 * i + 2];
        /* project.cpp:537-541 (R@mean, then + t in the per-Gaussian pass :559-561). */
        const float tx = (mx * r00 + my * r01 + mz * r02) + t0;
        const float ty = (mx * r10 + my * r11 + mz * r12) + t1;
        const float tz = (mx * r20 + my * r21 + mz * r22) + t2;
        if (tz <= 0.2f || (opacities != NULL && opacities[i] < min_opacity)) {
            valid_mask[i] = 0; /* :575-587 */
            continue;
        }
        const float inv_tz = 1.0f / tz;
        const float mean_x = fx * tx * inv_tz + cx;
        const float mean_y = fy * ty * inv_tz + cy;
        const float tz2 = tz * tz;
        const float j00 = fx / tz, j02 = -fx * tx / tz2;
        const float j11 = fy / tz, j12 = -fy * ty / tz2;
        const float* c3 = cov3d + 9 * i;
        const float c00 = c3[0], c01 = c3[1], c02 = c3[2], c11 = c3[4], c12 = c3[5], c22 = c3[8];
        /* :623-641 v_j = cov3d @ R(j,:)^T, cov_cam(i,j) = R(i,:) . v_j */
        const float v00 = c00 * r00 + c01 * r01 + c02 * r02;
        const float v01 = c01 * r00 + c11 * r01 + c12 * r02;
        const float v02 = c02 * r00 + c12 * r01 + c22 * r02;
        const float v10 = c00 * r10 + c01 * r11 + c02 * r12;
        const float v11 = c01 * r10 + c11 * r11 + c12 * r12;
        const float v12 = c02 * r10 + c12 * r11 + c22 * r12;
        const float v20 = c00 * r20 + c01 * r21 + c02 * r22;
        const float v21 = c01 * r20 + c11 * r21 + c12 * r22;
        const float v22 = c02 * r20 + c12 * r21 + c22 * r22;
        const float cc00 = r00 * v00 + r01 * v01 + r02 * v02;
        const float cc01 = r00 * v10 + r01 * v11 + r02 * v12;
        const float cc02 = r00 * v20 + r01 * v21 + r02 * v22;
        const float cc11 = r10 * v10 + r11 * v11 + r12 * v12;
        const float cc12 = r10 * v20 + r11 * v21 + r12 * v22;
        const float cc22 = r20 * v20 + r21 * v21 + r22 * v22;
        /* :646-653 cov2d = J cov_cam J^T + 0.3 I with the sparse J expanded. */
        const float m00 = j00 * cc00 + j02 * cc02;
        const float m01 = j00 * cc01 + j02 * cc12;
        const float m02 = j00 * cc02 + j02 * cc22;
        const float m11 = j11 * cc11 + j12 * cc12;
        const float m12 = j11 * cc12 + j12 * cc22;
        const float a = m00 * j00 + m02 * j02 + 0.3f;
        const float b = m01 * j11 + m02 * j12;
        const float c = m11 * j11 + m12 * j12 + 0.3f;
        /* :659-676 opacity-aware sigma multiplier, axis-aligned radii (isoellipse off). */
        float kk = opacities != NULL ? opacity_k(opacities[i], contrib_floor_k) : 3.0f;
        if (k_cap > 0.0f) kk = fminf_ref(kk, k_cap);
        const float rx = ceilf(kk * sqrtf(fmaxf_ref(a, 0.0f)));
        const float ry = ceilf(kk * sqrtf(fmaxf_ref(c, 0.0f)));
        /* :679-686 on-screen and radius tests. */
        const int ok = (mean_x + rx > 0.0f) && (mean_x - rx < (float)width) &&
                       (mean_y + ry > 0.0f) && (mean_y - ry < (float)height) && (rx > 0.0f) &&
                       (ry > 0.0f) && (rx <= max_r) && (ry <= max_r);
        valid_mask[i] = (uint8_t)ok;
        if (!ok) continue;
        /* :710-797 stable compaction in input order. */
        means_2d[2 * m] = mean_x;
        means_2d[2 * m + 1] = mean_y;
        covs_2d[4 * m] = a;
        covs_2d[4 * m + 1] = b;
        covs_2d[4 * m + 2] = b;
        covs_2d[4 * m + 3] = c;
        depths[m] = tz;
        radii[2 * m] = rx;
        radii[2 * m + 1] = ry;
        if (opacities != NULL && opacities_out != NULL) opacities_out[m] = opacities[i];
        if (colors != NULL && colors_out != NULL) {
            colors_out[3 * m] = colors[3 * i];
            colors_out[3 * m + 1] = colors[3 * i + 1];
            colors_out[3 * m + 2] = colors[3 * i + 2];
        }
        ++m;
    }
    return m;
}

int64_t gso_tile_assign(const float* means_2d, const float* radii, int64_t m, int height,
                        int width, int tile_size, const float* covs_2d, const float* opacities,
                        float contrib_floor, int64_t* gids, int64_t* tids, int64_t* tpg) {
    const int tiles_x = (width + tile_size - 1) / tile_size;
    const int tiles_y = (height + tile_size - 1) / tile_size;
    const float ts = (float)tile_size;
    /* tile_assign.cpp:60-86 rectangle; :107-111 exclusive prefix sum. */
    int64_t p = 0;
    for (int64_t g = 0; g < m; ++g) {
        const float px = means_2d[2 * g], py = means_2d[2 * g + 1];
        const float rx = radii[2 * g], ry = radii[2 * g + 1];
        const int x0 = clampi((int)((px - rx) / ts), 0, tiles_x - 1);
        const int x1 = clampi((int)((px + rx) / ts), 0, tiles_x - 1);
        const int y0 = clampi((int)((py - ry) / ts), 0, tiles_y - 1);
        const int y1 = clampi((int)((py + ry) / ts), 0, tiles_y - 1);
        const int64_t cnt = (int64_t)(x1 - x0 + 1) * (int64_t)(y1 - y0 + 1);
        if (tpg != NULL) tpg[g] = cnt;
        if (gids != NULL) {
            /* :121-135 Gaussian-major, row-major pair emission. */
            int64_t pos = p;
            for (int y = y0; y <= y1; ++y)
                for (int x = x0; x <= x1; ++x) {
                    gids[pos] = g;
                    tids[pos] = (int64_t)y * tiles_x + x;
                    ++pos;
                }
        }
        p += cnt;
    }
    if (gids == NULL || covs_2d == NULL || opacities == NULL || p == 0) return p;

    /* :151-350 exact min-Mahalanobis cull of each pair against contrib_floor, then an
     * order-preserving compaction and a recount of tiles_per_gaussian. */
    int64_t out = 0;
    for (int64_t i = 0; i < p; ++i) {
        const int64_t g = gids[i];
        const int64_t tile = tids[i];
        const float op = opacities[g];
        int keep;
        if (!(op > contrib_floor)) {
            keep = 0;
        } else {
            const float thresh = -2.0f * logf(contrib_floor / op);
            const float a = covs_2d[4 * g], b = covs_2d[4 * g + 1], c = covs_2d[4 * g + 3];
            const float det = fmaxf_ref(a * c - b * b, 1e-6f);
            const float px = means_2d[2 * g], py = means_2d[2 * g + 1];
            const float tx0 = (float)(tile % tiles_x) * ts;
            const float ty0 = (float)(tile / tiles_x) * ts;
            const float u_lo = tx0 - px, u_hi = u_lo + ts;
            const float v_lo = ty0 - py, v_hi = v_lo + ts;
            const int x_in = (u_lo <= 0.0f) && (0.0f <= u_hi);
            const int y_in = (v_lo <= 0.0f) && (0.0f <= v_hi);
            const float scaled = det * thresh;
            if (x_in && y_in) {
                keep = 1;
            } else {
                float m2v = INFINITY, m2h = INFINITY;
                if (!x_in) {
                    const float uf = (u_lo > 0.0f) ? u_lo : u_hi;
                    float vs = (b * uf) / fmaxf_ref(a, 1e-12f);
                    vs = fmaxf_ref(v_lo, fminf_ref(vs, v_hi));
                    m2v = c * uf * uf - 2.0f * b * uf * vs + a * vs * vs;
                }
                if (!y_in) {
                    const float vf = (v_lo > 0.0f) ? v_lo : v_hi;
                    float us = (b * vf) / fmaxf_ref(c, 1e-12f);
                    us = fmaxf_ref(u_lo, fminf_ref(us, u_hi));
                    m2h = c * us * us - 2.0f * b * us * vf + a * vf * vf;
                }
                keep = fminf_ref(m2v, m2h) <= scaled;
            }
        }
        if (keep) {
            gids[out] = g;
            tids[out] = tile;
            ++out;
        }
    }
    if (tpg != NULL) {
        memset(tpg, 0, (size_t)m * sizeof(int64_t));
        for (int64_t i = 0; i < out; ++i) tpg[gids[i]] += 1;
    }
    return out;
}

/* Stable LSD radix sort over 16-bit digits of the 64-bit keys. */
void gso_sort_pairs(const uint64_t* keys, const uint32_t* values, int64_t n, uint64_t* keys_out,
                    uint32_t* values_out) {
    if (n <= 0) return;
    uint64_t* ka = (uint64_t*)malloc((size_t)n * 8);
    uint32_t* va = (uint32_t*)malloc((size_t)n * 4);
    uint64_t* kb = (uint64_t*)malloc((size_t)n * 8);
    uint32_t* vb = (uint32_t*)malloc((size_t)n * 4);
    size_t* cnt = (size_t*)malloc(65536 * sizeof(size_t));
    memcpy(ka, keys, (size_t)n * 8);
    memcpy(va, values, (size_t)n * 4);
    uint64_t all_or = 0;
    for (int64_t i = 0; i < n; ++i) all_or |= ka[i];
    for (int shift = 0; shift < 64; shift += 16) {
        if ((all_or >> shift) == 0) break; /* remaining digits are all zero */
        memset(cnt, 0, 65536 * sizeof(size_t));
        for (int64_t i = 0; i < n; ++i) cnt[(ka[i] >> shift) & 0xFFFF]++;
        size_t s = 0;
        for (int d = 0; d < 65536; ++d) {
            const size_t c = cnt[d];
            cnt[d] = s;
            s += c;
        }
        for (int64_t i = 0; i < n; ++i) {
            const size_t pos = cnt[(ka[i] >> shift) & 0xFFFF]++;
            kb[pos] = ka[i];
            vb[pos] = va[i];
        }
        uint64_t* tk = ka; ka = kb; kb = tk;
        uint32_t* tv = va; va = vb; vb = tv;
    }
    memcpy(keys_out, ka, (size_t)n * 8);
    memcpy(values_out, va, (size_t)n * 4);
    free(ka); free(va); free(kb); free(vb); free(cnt);
}

void gso_sort_and_bin(const int64_t* gids, const int64_t* tids, const float* depths, int64_t p,
                      int tiles_x, int tiles_y, int64_t* sorted, int64_t* ranges) {
    const int64_t nt = (int64_t)tiles_x * tiles_y;
    memset(ranges, 0, (size_t)nt * 2 * sizeof(int64_t));
    if (p <= 0) return;
    /* sort.cpp:124-205 stable bin by tile, :207-257 stable depth-bit sort per tile:
     * together a stable sort on key = tile << 32 | bits(depth). Values are pair
     * positions so 64-bit Gaussian ids pass through unchanged. */
    uint64_t* keys = (uint64_t*)malloc((size_t)p * 8);
    uint32_t* pos = (uint32_t*)malloc((size_t)p * 4);
    uint64_t* ks = (uint64_t*)malloc((size_t)p * 8);
    uint32_t* ps = (uint32_t*)malloc((size_t)p * 4);
    for (int64_t i = 0; i < p; ++i) {
        uint32_t bits;
        memcpy(&bits, &depths[gids[i]], 4);
        keys[i] = ((uint64_t)tids[i] << 32) | bits;
        pos[i] = (uint32_t)i;
    }
    gso_sort_pairs(keys, pos, p, ks, ps);
    for (int64_t i = 0; i < p; ++i) sorted[i] = gids[ps[i]];
    /* :146-165 ranges [start, end) per populated tile, (0, 0) for empty tiles. */
    for (int64_t i = 0; i < p; ++i) {
        const int64_t t = (int64_t)(ks[i] >> 32);
        if (i == 0 || (int64_t)(ks[i - 1] >> 32) != t) ranges[2 * t] = i;
        if (i == p - 1 || (int64_t)(ks[i + 1] >> 32) != t) ranges[2 * t + 1] = i + 1;
    }
    free(keys); free(pos); free(ks); free(ps);
}

void gso_blend(const float* means_2d, const float* covs_2d, const float* colors,
               const float* opacities, const int64_t* sorted, const int64_t* ranges, int64_t m,
               int height, int width, int tile_size, float* image, float* alpha_out) {
    const int tiles_x = (width + tile_size - 1) / tile_size;
    const int tiles_y = (height + tile_size - 1) / tile_size;
    memset(image, 0, (size_t)height * width * 3 * sizeof(float));
    if (alpha_out != NULL) memset(alpha_out, 0, (size_t)height * width * sizeof(float));
    /* blend.cpp:136-146 conic with the determinant clamp. */
    float* inv = (float*)malloc((size_t)(m > 0 ? m : 1) * 3 * sizeof(float));
    for (int64_t i = 0; i < m; ++i) {
        const float a = covs_2d[4 * i], b = covs_2d[4 * i + 1], c = covs_2d[4 * i + 3];
        const float det = fmaxf_ref(a * c - b * b, 1e-6f);
        inv[3 * i] = c / det;
        inv[3 * i + 1] = -b / det;
        inv[3 * i + 2] = a / det;
    }
    float T[32 * 32], acc[32 * 32 * 3];
    for (int tile = 0; tile < tiles_x * tiles_y; ++tile) {
        const int64_t start = ranges[2 * tile], end = ranges[2 * tile + 1];
        if (start == end) continue;
        const int ty = tile / tiles_x, tx = tile % tiles_x;
        const int y0 = ty * tile_size, x0 = tx * tile_size;
        const int th = (y0 + tile_size < height ? y0 + tile_size : height) - y0;
        const int tw = (x0 + tile_size < width ? x0 + tile_size : width) - x0;
        for (int k = 0; k < th * tw; ++k) {
            T[k] = 1.0f;
            acc[3 * k] = acc[3 * k + 1] = acc[3 * k + 2] = 0.0f;
        }
        /* blend.cpp:58-94 front to back over the tile's sorted pairs. */
        for (int64_t idx = start; idx < end; ++idx) {
            const int64_t g = sorted[idx];
            const float ia = inv[3 * g], ib = inv[3 * g + 1], ic = inv[3 * g + 2];
            const float mx = means_2d[2 * g], my = means_2d[2 * g + 1];
            const float op = opacities[g];
            const float cr = colors[3 * g], cg = colors[3 * g + 1], cb = colors[3 * g + 2];
            for (int i = 0; i < th; ++i) {
                const float py = (float)(y0 + i) + 0.5f;
                for (int j = 0; j < tw; ++j) {
                    const float px = (float)(x0 + j) + 0.5f;
                    const float dx = px - mx, dy = py - my;
                    const float power = -0.5f * (ia * dx * dx + 2.0f * ib * dx * dy + ic * dy * dy);
                    const float gw = expf(fminf_ref(power, 0.0f));
                    const float alpha = fminf_ref(op * gw, 0.99f);
                    const int q = i * tw + j;
                    const float t = T[q];
                    const float at = alpha * t;
                    acc[3 * q] += at * cr;
                    acc[3 * q + 1] += at * cg;
                    acc[3 * q + 2] += at * cb;
                    T[q] = t * (1.0f - alpha);
                }
            }
            float tmax = 0.0f;
            for (int q = 0; q < th * tw; ++q) tmax = fmaxf_ref(tmax, T[q]);
            if (tmax < 0.0001f) break; /* tile-level stop */
        }
        for (int i = 0; i < th; ++i)
            for (int j = 0; j < tw; ++j) {
                const int q = i * tw + j;
                const size_t o = (size_t)(y0 + i) * width + (x0 + j);
                image[3 * o] = acc[3 * q];
                image[3 * o + 1] = acc[3 * q + 1];
                image[3 * o + 2] = acc[3 * q + 2];
                if (alpha_out != NULL) alpha_out[o] = 1.0f - T[q];
            }
    }
    free(inv);
}

/* ---------------------------------------------------------------- microblock cull + blend
 * src/gsplat_cpu/cull_and_blend.cpp:316-840 cull_and_blend as the reference's scalar build
 * runs it (no GSPLAT_SIMD_AVX2 / NEON: every microblock goes through the scalar blend loop).
 * A tile is cut into 8x4-pixel microblocks, mb = (my << 2) | mx for mx 0..3, my 0..7;
 * per Gaussian of the tile list (sorted order): drop if opacity <= mb_contrib_floor or
 * its opacity-scaled bounding box misses every microblock; else keep it in each
 * microblock whose exact minimum Mahalanobis distance over the microblock rectangle
 * reaches the floor (cull.cpp:408-475). Each microblock then blends its kept list in order
 * with alpha = min(op * exp(min(power, 0)), 0.99) and stops after the first Gaussian that
 * leaves every pixel's T below transmittance_threshold (:599-640). */
typedef struct {
    float mx, my, ia, ib, ic, lt, xh, yh, op, r, g, b;
} CullRec;

static float clampf_ref(float v, float lo, float hi) { return v < lo ? lo : (hi < v ? hi : v); }

void gso_cull_and_blend(const float* means_2d, const float* covs_2d, const float* colors,
                        const float* opacities, const int64_t* sorted_ids,
                        const int64_t* tile_ranges, int64_t m, int64_t p, int tiles_x,
                        int tiles_y, int tile_size, int height, int width,
                        float mb_contrib_floor, int cull_disabled,
                        float transmittance_threshold, float* image, int64_t* stats) {
    CullRec* rec = (CullRec*)malloc((size_t)(m > 0 ? m : 1) * sizeof(CullRec));
    for (int64_t i = 0; i < m; ++i) {
        const float a = covs_2d[4 * i], b = covs_2d[4 * i + 1], c = covs_2d[4 * i + 3];
        const float det = fmaxf_ref(a * c - b * b, 1e-6f);
        CullRec* r = &rec[i];
        r->mx = means_2d[2 * i];
        r->my = means_2d[2 * i + 1];
        r->ia = c / det;
        r->ib = -b / det;
        r->ic = a / det;
        r->op = opacities[i];
        r->r = colors[3 * i];
        r->g = colors[3 * i + 1];
        r->b = colors[3 * i + 2];
        if (r->op <= mb_contrib_floor) {
            r->lt = 0.0f;
            r->xh = r->yh = 0.0f;
        } else {
            r->lt = logf(mb_contrib_floor / r->op);
            const float rd = sqrtf(-2.0f * r->lt);
            r->xh = rd * sqrtf(fmaxf_ref(a, 0.0f));
            r->yh = rd * sqrtf(fmaxf_ref(c, 0.0f));
        }
    }
    int64_t dropped = 0, kept = 0;
    int64_t lmax = 0;
    for (int t = 0; t < tiles_x * tiles_y; ++t) {
        const int64_t L = tile_ranges[2 * t + 1] - tile_ranges[2 * t];
        if (L > lmax) lmax = L;
    }
    int64_t* lists = (int64_t*)malloc((size_t)(32 * (lmax > 0 ? lmax : 1)) * sizeof(int64_t));
    for (int t = 0; t < tiles_x * tiles_y; ++t) {
        const int64_t start = tile_ranges[2 * t], end = tile_ranges[2 * t + 1];
        if (start == end) continue;
        const int ty = t / tiles_x, tx = t % tiles_x;
        const float txt = (float)(tx * tile_size), tyt = (float)(ty * tile_size);
        const int py_tile = ty * tile_size, px_tile = tx * tile_size;
        const int py_end_tile = py_tile + tile_size < height ? py_tile + tile_size : height;
        const int px_end_tile = px_tile + tile_size < width ? px_tile + tile_size : width;
        const int64_t L = end - start;
        int64_t cnt[32];
        for (int q = 0; q < 32; ++q) cnt[q] = 0;
        for (int64_t l = 0; l < L; ++l) {
            const int64_t g = sorted_ids[start + l];
            const CullRec* r = &rec[g];
            if (r->lt >= 0.0f) {
                ++dropped;
                continue;
            }
            const int mx_lo = clampi((int)floorf(((r->mx - r->xh) - txt) / 8.0f), 0, 1 << 30);
            const int mx_hi_raw = (int)floorf(((r->mx + r->xh) - txt) / 8.0f);
            const int my_lo = clampi((int)floorf(((r->my - r->yh) - tyt) / 4.0f), 0, 1 << 30);
            const int my_hi_raw = (int)floorf(((r->my + r->yh) - tyt) / 4.0f);
            const int mx_hi = mx_hi_raw < 3 ? mx_hi_raw : 3;
            const int my_hi = my_hi_raw < 7 ? my_hi_raw : 7;
            if (mx_lo > mx_hi || my_lo > my_hi) {
                ++dropped;
                continue;
            }
            const float thresh = -2.0f * r->lt;
            const float ia_s = fmaxf_ref(r->ia, 1e-12f), ic_s = fmaxf_ref(r->ic, 1e-12f);
            int any = 0;
            for (int my = my_lo; my <= my_hi; ++my) {
                const float v_lo = (tyt + (float)(my * 4)) - r->my;
                const float v_hi = v_lo + 4.0f;
                const int y_in = (v_lo <= 0.0f) && (0.0f <= v_hi);
                const float v_fix = (v_lo > 0.0f) ? v_lo : v_hi;
                for (int mx = mx_lo; mx <= mx_hi; ++mx) {
                    const float u_lo = (txt + (float)(mx * 8)) - r->mx;
                    const float u_hi = u_lo + 8.0f;
                    const int x_in = (u_lo <= 0.0f) && (0.0f <= u_hi);
                    float m2;
                    if (cull_disabled || (x_in && y_in)) {
                        m2 = 0.0f;
                    } else {
                        float m2v = INFINITY, m2h = INFINITY;
                        if (!x_in) {
                            const float uf = (u_lo > 0.0f) ? u_lo : u_hi;
                            const float vs = clampf_ref(-r->ib * uf / ic_s, v_lo, v_hi);
                            m2v = r->ia * uf * uf + 2.0f * r->ib * uf * vs + r->ic * vs * vs;
                        }
                        if (!y_in) {
                            const float us = clampf_ref(-r->ib * v_fix / ia_s, u_lo, u_hi);
                            m2h = r->ia * us * us + 2.0f * r->ib * us * v_fix + r->ic * v_fix * v_fix;
                        }
                        m2 = fminf_ref(m2v, m2h);
                    }
                    if (m2 <= thresh) {
                        const int mb = (my << 2) | mx;
                        lists[mb * lmax + cnt[mb]++] = g;
                        any = 1;
                        ++kept;
                    }
                }
            }
            if (!any) ++dropped;
        }
        for (int mb = 0; mb < 32; ++mb) {
            if (cnt[mb] == 0) continue;
            const int py0 = py_tile + (mb >> 2) * 4, px0 = px_tile + (mb & 3) * 8;
            const int py1 = py0 + 4 < py_end_tile ? py0 + 4 : py_end_tile;
            const int px1 = px0 + 8 < px_end_tile ? px0 + 8 : px_end_tile;
            if (py0 >= py1 || px0 >= px1) continue;
            const int h = py1 - py0, w = px1 - px0;
            float T[32], acc[96];
            for (int q = 0; q < h * w; ++q) T[q] = 1.0f;
            for (int q = 0; q < 3 * h * w; ++q) acc[q] = 0.0f;
            for (int64_t k = 0; k < cnt[mb]; ++k) {
                const CullRec* r = &rec[lists[mb * lmax + k]];
                for (int i = 0; i < h; ++i) {
                    const float py = (float)(py0 + i) + 0.5f;
                    for (int j = 0; j < w; ++j) {
                        const float px = (float)(px0 + j) + 0.5f;
                        const float dx = px - r->mx, dy = py - r->my;
                        const float power =
                            -0.5f * (r->ia * dx * dx + 2.0f * r->ib * dx * dy + r->ic * dy * dy);
                        const float gw = expf(fminf_ref(power, 0.0f));
                        const float alpha = fminf_ref(r->op * gw, 0.99f);
                        const int q = i * w + j;
                        const float tq = T[q];
                        const float at = alpha * tq;
                        acc[3 * q] += at * r->r;
                        acc[3 * q + 1] += at * r->g;
                        acc[3 * q + 2] += at * r->b;
                        T[q] = tq * (1.0f - alpha);
                    }
                }
                float tmax = 0.0f;
                for (int q = 0; q < h * w; ++q) tmax = fmaxf_ref(tmax, T[q]);
                if (tmax < transmittance_threshold) break;
            }
            for (int i = 0; i < h; ++i)
                for (int j = 0; j < w; ++j) {
                    const int q = i * w + j;
                    const size_t o = (size_t)(py0 + i) * width + (px0 + j);
                    image[3 * o] = acc[3 * q];
                    image[3 * o + 1] = acc[3 * q + 1];
                    image[3 * o + 2] = acc[3 * q + 2];
                }
        }
    }
    stats[0] = p;
    stats[1] = dropped;
    stats[2] = kept;
    free(lists);
    free(rec);
}

/* Host C library logf over an array (checker for the device reproduction). */
void gso_logf_array(const float* x, float* y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = logf(x[i]);
}
