/*
 * CPU oracle for the volume-integration renderer -- TEST INFRASTRUCTURE ONLY.
 *
 * This file restates, in scalar C, the algorithm of the reference extension
 * (NilKel/volume-integration, paths below are relative to that project).  It is
 * the checker for the CUDA path: only tests/, __graft_entry__.smoke() and the
 * cpu_baseline / reference arm of bench.py load it.  Nothing in the product
 * library links or calls it.
 *
 * Semantics restated ("program order"):
 *   - preprocess          cuda_integrator/forward.cu:27-110, auxiliary.h:50-86,148-175
 *   - offsets scan        cuda_integrator/integrator_impl.cu:306
 *   - duplicateWithKeys   cuda_integrator/integrator_impl.cu:106-147
 *   - radix sort          cuda_integrator/integrator_impl.cu:341-349 (CUB stable LSD sort
 *                         over bits [0, 32+getHigherMsb(tiles)); restated as a stable
 *                         counting sort, which yields the same permutation)
 *   - identifyTileRanges  cuda_integrator/integrator_impl.cu:152-178
 *   - renderCUDA<3>       cuda_integrator/forward.cu:146-792, hashgrid.h:207-299
 *   - unifiedBackward<3>  cuda_integrator/backward.cu:51-792, hashgrid.h:9-96
 *   - checkFrustum        cuda_integrator/integrator_impl.cu:66-78
 *
 * The reference render kernel executes a CTA barrier that pixels with no
 * covering grid point skip (forward.cu:629-631 `continue` vs the barrier at
 * forward.cu:715).  Its GPU output is therefore schedule dependent.  This oracle
 * defines the behaviour each pixel thread would have if every barrier were
 * reached in order: each pixel walks its tile's list in order and sees, for
 * each entry, that entry's own stage-1 data.
 *
 * Floating point: compiled with -ffp-contract=off, so every a*b+c is two
 * roundings.  Where the reference uses double literals (ndc2Pix, the 1e-6 in
 * the radius) the arithmetic is done in double exactly as C promotes it.
 *
 * Defined behaviour where the reference is undefined (stated once here):
 *   - a visible primitive whose integer radius is <= 0 is culled; the reference
 *     reserves tiles for it but never writes those keys (integrator_impl.cu:121).
 *   - the linear layer is W[o*D + i] with D = L*F (the reference reads stride 32,
 *     forward.cu:457, which equals D only when D == 32, its only well-defined case).
 *   - no compile-time caps: D, O and G are runtime sizes (the reference caps them
 *     at 32, 8 and 5, forward.cu:201-216).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <limits.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define TILE 16

typedef struct { float x, y; } f2;
typedef struct { float x, y, z; } f3;

/* float -> int32 conversion with the GPU's cvt.rzi.s32.f32 behaviour
 * (truncate, saturate, NaN -> 0). */
static int f2i_rz(float x) {
    if (x != x) return 0;
    if (x >= 2147483648.0f) return INT_MAX;
    if (x <= -2147483648.0f) return INT_MIN;
    return (int)x;
}

/* auxiliary.h:67-75 */
static f3 t43(f3 p, const float *m) {
    f3 r;
    r.x = m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12];
    r.y = m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13];
    r.z = m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14];
    return r;
}

/* auxiliary.h:77-86 */
static void t44(f3 p, const float *m, float *o) {
    o[0] = m[0] * p.x + m[4] * p.y + m[8] * p.z + m[12];
    o[1] = m[1] * p.x + m[5] * p.y + m[9] * p.z + m[13];
    o[2] = m[2] * p.x + m[6] * p.y + m[10] * p.z + m[14];
    o[3] = m[3] * p.x + m[7] * p.y + m[11] * p.z + m[15];
}

/* auxiliary.h:50-53: ((v + 1.0) * S - 1.0) * 0.5, evaluated in double. */
static float ndc2pix(float v, int S) {
    return (float)((((double)v + 1.0) * (double)S - 1.0) * 0.5);
}

/* auxiliary.h:55-65 */
static void get_rect(f2 p, int r, unsigned gx, unsigned gy,
                     unsigned *minx, unsigned *miny, unsigned *maxx, unsigned *maxy) {
    float rf = (float)r;
    int a;
    a = f2i_rz((p.x - rf) / (float)TILE); a = a > 0 ? a : 0; *minx = (unsigned)a < gx ? (unsigned)a : gx;
    a = f2i_rz((p.y - rf) / (float)TILE); a = a > 0 ? a : 0; *miny = (unsigned)a < gy ? (unsigned)a : gy;
    a = f2i_rz((p.x + rf + (float)TILE - 1.0f) / (float)TILE); a = a > 0 ? a : 0; *maxx = (unsigned)a < gx ? (unsigned)a : gx;
    a = f2i_rz((p.y + rf + (float)TILE - 1.0f) / (float)TILE); a = a > 0 ? a : 0; *maxy = (unsigned)a < gy ? (unsigned)a : gy;
}

/* integrator_impl.cu:47-62 */
unsigned vio_higher_msb(unsigned n) {
    unsigned msb = sizeof(n) * 4, step = msb;
    while (step > 1) {
        step /= 2;
        if (n >> msb) msb += step; else msb -= step;
    }
    if (n >> msb) msb++;
    return msb;
}

/* ------------------------------------------------------------------------ */
/* R1: preprocess (forward.cu:27-110, in_frustum auxiliary.h:148-175)          */
/* ------------------------------------------------------------------------ */
void vio_preprocess(int P, const float *means, float scale, const float *view, const float *proj,
                    int W, int H, float tanfovx, float tanfovy,
                    int *radii, float *means2D, float *depths, uint32_t *tiles_touched) {
    unsigned gx = (W + TILE - 1) / TILE, gy = (H + TILE - 1) / TILE;
    float focal_y = (float)H / (2.0f * tanfovy);   /* integrator_impl.cu:273-274 */
    float focal_x = (float)W / (2.0f * tanfovx);
    for (int i = 0; i < P; i++) {
        radii[i] = 0;
        tiles_touched[i] = 0;
        f3 p = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
        f3 pv = t43(p, view);
        if (pv.z <= 0.2f) continue;
        float ph[4];
        t44(p, proj, ph);
        float pw = 1.0f / (ph[3] + 0.0000001f);
        float px = ph[0] * pw, py = ph[1] * pw;
        float world_radius = scale * 0.86602540378f;
        float view_depth = (float)((double)fabsf(pv.z) + 1e-6);
        float srx = world_radius * focal_x / view_depth;
        float sry = world_radius * focal_y / view_depth;
        int r = f2i_rz(ceilf(fmaxf(srx, sry)));
        f2 img = {ndc2pix(px, W), ndc2pix(py, H)};
        unsigned x0, y0, x1, y1;
        get_rect(img, r, gx, gy, &x0, &y0, &x1, &y1);
        if ((x1 - x0) * (y1 - y0) == 0) continue;
        if (r <= 0) continue; /* defined behaviour, see header */
        depths[i] = pv.z;
        radii[i] = r;
        means2D[2 * i] = img.x;
        means2D[2 * i + 1] = img.y;
        tiles_touched[i] = (y1 - y0) * (x1 - x0);
    }
}

/* R2: inclusive scan (integrator_impl.cu:306); returns the total. */
uint64_t vio_scan(int P, const uint32_t *tt, uint32_t *offsets) {
    uint32_t acc = 0;
    uint64_t tot = 0;
    for (int i = 0; i < P; i++) { acc += tt[i]; tot += tt[i]; offsets[i] = acc; }
    return tot;
}

/* R3: duplicateWithKeys (integrator_impl.cu:106-147) */
void vio_duplicate(int P, const float *means2D, const float *depths, const uint32_t *offsets,
                   const int *radii, int W, int H, uint64_t *keys, uint32_t *vals) {
    unsigned gx = (W + TILE - 1) / TILE, gy = (H + TILE - 1) / TILE;
    for (int i = 0; i < P; i++) {
        if (radii[i] <= 0) continue;
        uint32_t off = i == 0 ? 0 : offsets[i - 1];
        unsigned x0, y0, x1, y1;
        f2 p = {means2D[2 * i], means2D[2 * i + 1]};
        get_rect(p, radii[i], gx, gy, &x0, &y0, &x1, &y1);
        uint32_t dbits;
        memcpy(&dbits, &depths[i], 4);
        for (unsigned y = y0; y < y1; y++)
            for (unsigned x = x0; x < x1; x++) {
                uint64_t k = (uint64_t)(y * gx + x);
                keys[off] = (k << 32) | dbits;
                vals[off] = (uint32_t)i;
                off++;
            }
    }
}

/* R4: stable LSD sort over bits [0,end_bit), 8-bit digits (same permutation as
 * cub::DeviceRadixSort::SortPairs, which is stable). */
void vio_sort(uint64_t R, const uint64_t *kin, const uint32_t *vin, uint64_t *kout, uint32_t *vout,
              int end_bit) {
    uint64_t *ka = malloc(R * 8 + 8), *kb = malloc(R * 8 + 8);
    uint32_t *va = malloc(R * 4 + 4), *vb = malloc(R * 4 + 4);
    memcpy(ka, kin, R * 8);
    memcpy(va, vin, R * 4);
    for (int shift = 0; shift < end_bit; shift += 8) {
        int bits = end_bit - shift < 8 ? end_bit - shift : 8;
        uint64_t mask = (1ull << bits) - 1;
        uint64_t cnt[257];
        memset(cnt, 0, sizeof cnt);
        for (uint64_t i = 0; i < R; i++) cnt[((ka[i] >> shift) & mask) + 1]++;
        for (int d = 0; d < 256; d++) cnt[d + 1] += cnt[d];
        for (uint64_t i = 0; i < R; i++) {
            uint64_t d = (ka[i] >> shift) & mask;
            uint64_t o = cnt[d]++;
            kb[o] = ka[i];
            vb[o] = va[i];
        }
        uint64_t *tk = ka; ka = kb; kb = tk;
        uint32_t *tv = va; va = vb; vb = tv;
    }
    memcpy(kout, ka, R * 8);
    memcpy(vout, va, R * 4);
    free(ka); free(kb); free(va); free(vb);
}

/* R6: identifyTileRanges (integrator_impl.cu:152-178); ranges pre-zeroed by the
 * caller as the reference memsets them (integrator_impl.cu:355). */
void vio_ranges(uint64_t R, const uint64_t *keys, uint32_t *ranges /* 2 per tile */) {
    for (uint64_t i = 0; i < R; i++) {
        uint32_t cur = (uint32_t)(keys[i] >> 32);
        if (i == 0) ranges[2 * cur] = 0;
        else {
            uint32_t prev = (uint32_t)(keys[i - 1] >> 32);
            if (cur != prev) { ranges[2 * prev + 1] = (uint32_t)i; ranges[2 * cur] = (uint32_t)i; }
        }
        if (i == R - 1) ranges[2 * cur + 1] = (uint32_t)R;
    }
}

/* checkFrustum (integrator_impl.cu:66-78) */
void vio_mark_visible(int P, const float *means, const float *view, uint8_t *present) {
    for (int i = 0; i < P; i++) {
        f3 p = {means[3 * i], means[3 * i + 1], means[3 * i + 2]};
        present[i] = t43(p, view).z <= 0.2f ? 0 : 1;
    }
}

/* ------------------------------------------------------------------------ */
/* Stage 1 shared by render and backward                                     */
/* ------------------------------------------------------------------------ */
typedef struct {
    int P, W, H;
    const float *means, *conf;
    float scale;
    const float *view, *proj;
    float near_plane, max_distance;
    const float *table;
    const int *res, *do_hash, *primes;
    int T;
    const float *Wl, *bl;
    int genus, G, K;
    const float *bg;
    int F, Fout, L;
    uint64_t table_size; /* feature_table.numel(), backward bound check hashgrid.h:88 */
    float hlo[3], hext[3]; /* hashgrid box: lower corner, extent; the reference fixes -1.3, 2.6 (hashgrid.h:23-24) */
} vio_params;

/* Table entry index of one corner, or -1 (hashgrid.h:258-275 / :57-74). */
static int64_t corner_entry(int cx, int cy, int cz, int res, int use_hash, const int *primes, int T) {
    if (use_hash) {
        uint32_t h = 0;
        h ^= (uint32_t)cx * (uint32_t)primes[0];
        h ^= (uint32_t)cy * (uint32_t)primes[1];
        h ^= (uint32_t)cz * (uint32_t)primes[2];
        return (int64_t)(h % (uint32_t)T);
    }
    if (cx < 0 || cx >= res || cy < 0 || cy >= res || cz < 0 || cz >= res) return -1;
    uint32_t e = (uint32_t)cz * (uint32_t)res * (uint32_t)res + (uint32_t)cy * (uint32_t)res + (uint32_t)cx;
    if (e >= (uint32_t)T) return -1;
    return (int64_t)e;
}

/* Level setup common to interpolation and gradient (hashgrid.h:225-242). */
static void level_setup(const vio_params *p, f3 pos, int res, int *base, float *t) {
    float n[3] = {(pos.x - p->hlo[0]) / p->hext[0], (pos.y - p->hlo[1]) / p->hext[1],
                  (pos.z - p->hlo[2]) / p->hext[2]};
    for (int a = 0; a < 3; a++) {
        float v = fmaxf(0.0f, fminf(1.0f, n[a]));
        float pl = v * (float)res;
        float fl = floorf(pl);
        base[a] = (int)fl;
        t[a] = pl - fl;
    }
}

/* hashInterpolateShared (hashgrid.h:207-299): writes phi[l*F+f] for f<F. */
static void hash_interp(const vio_params *p, f3 pos, int l, float *phi) {
    int res = p->res[l], b[3];
    float t[3];
    level_setup(p, pos, res, b, t);
    for (int f = 0; f < p->F; f++) {
        float acc = 0.0f;
        for (int dx = 0; dx < 2; dx++) {
            float wx = dx == 0 ? 1.0f - t[0] : t[0];
            for (int dy = 0; dy < 2; dy++) {
                float wy = dy == 0 ? 1.0f - t[1] : t[1];
                for (int dz = 0; dz < 2; dz++) {
                    float wz = dz == 0 ? 1.0f - t[2] : t[2];
                    float w = wx * wy * wz;
                    int64_t e = corner_entry(b[0] + dx, b[1] + dy, b[2] + dz, res, p->do_hash[l], p->primes, p->T);
                    if (e >= 0) acc += p->table[((uint64_t)e * p->L + l) * p->F + f] * w;
                }
            }
        }
        phi[l * p->F + f] = acc;
    }
}

/* hashComputeGradient (hashgrid.h:9-96): dz, dy, dx order, bound-checked. */
static void hash_grad(const vio_params *p, f3 pos, int l, const float *dphi, float *dtable, int threaded) {
    int res = p->res[l], b[3];
    float t[3];
    level_setup(p, pos, res, b, t);
    for (int dz = 0; dz < 2; dz++)
        for (int dy = 0; dy < 2; dy++)
            for (int dx = 0; dx < 2; dx++) {
                float w = 1.0f;
                w *= dx == 1 ? t[0] : 1.0f - t[0];
                w *= dy == 1 ? t[1] : 1.0f - t[1];
                w *= dz == 1 ? t[2] : 1.0f - t[2];
                int64_t e = corner_entry(b[0] + dx, b[1] + dy, b[2] + dz, res, p->do_hash[l], p->primes, p->T);
                if (e < 0) continue;
                uint64_t base = ((uint64_t)e * p->L + l) * p->F;
                for (int f = 0; f < p->F; f++) {
                    float v = dphi[f] * w;
                    if (base + f < p->table_size) {
                        if (threaded) {
#pragma omp atomic
                            dtable[base + f] += v;
                        } else dtable[base + f] += v;
                    }
                }
            }
}

/* Stage 1 for one primitive (forward.cu:401-463 / backward.cu:297-358).
 * fwd selects 1/(w+1e-7) (forward.cu:432) vs 1/w (backward.cu:325). */
static void stage1(const vio_params *p, uint32_t q, int fwd, float *conf, f2 *scr, float *phi, float *mlp) {
    int G = p->G, V = G * G * G, D = p->L * p->F, O = 3 + p->Fout + 1;
    f3 c = {p->means[3 * q], p->means[3 * q + 1], p->means[3 * q + 2]};
    float step = G > 1 ? p->scale / (float)(G - 1) : p->scale;
    float gof = (float)(G - 1) / 2.0f;
    for (int g = 0; g < V; g++) {
        conf[g] = p->conf[(uint64_t)q * V + g];
        int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G;
        float rx = ((float)x - gof) * step, ry = ((float)y - gof) * step, rz = ((float)z - gof) * step;
        f3 pos = {c.x + rx, c.y + ry, c.z + rz};
        float h[4];
        t44(pos, p->proj, h);
        float pw = fwd ? 1.0f / (h[3] + 0.0000001f) : 1.0f / h[3];
        scr[g].x = ndc2pix(h[0] * pw, p->W);
        scr[g].y = ndc2pix(h[1] * pw, p->H);
        float *ph = phi + (size_t)g * D;
        for (int i = 0; i < D; i++) ph[i] = 0.0f;
        for (int l = 0; l < p->L; l++) hash_interp(p, pos, l, ph);
        for (int o = 0; o < O; o++) {
            float s = 0.0f;
            for (int i = 0; i < D; i++) s += p->Wl[o * D + i] * ph[i];
            mlp[(size_t)g * O + o] = s;
        }
    }
}

static void stencil(int genus, int *S, float *c) {
    if (genus == 2) {
        *S = 5;
        c[0] = 1.0f / 12.0f; c[1] = -2.0f / 3.0f; c[2] = 0.0f; c[3] = 2.0f / 3.0f; c[4] = -1.0f / 12.0f;
    } else {
        *S = 3;
        c[0] = -0.5f; c[1] = 0.0f; c[2] = 0.5f;
    }
}

static int in_pixel(f2 s, unsigned px, unsigned py) {
    return s.x >= (float)px && s.x < ((float)px + 1.0f) && s.y >= (float)py && s.y < ((float)py + 1.0f);
}

/* Forward occupancy magnitude: neighbours count when conf > 0 (forward.cu:557-611). */
static float occ_mag_conf(const float *conf, int G, int g, int S, const float *cf) {
    int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G, off = (S - 1) / 2;
    float gx = 0.0f, gy = 0.0f, gz = 0.0f;
    for (int s = 0; s < S; s++) {
        int r = s - off, n;
        n = x + r; if (n >= 0 && n < G && conf[z * G * G + y * G + n] > 0.0f) gx += cf[s];
        n = y + r; if (n >= 0 && n < G && conf[z * G * G + n * G + x] > 0.0f) gy += cf[s];
        n = z + r; if (n >= 0 && n < G && conf[n * G * G + y * G + x] > 0.0f) gz += cf[s];
    }
    return fabsf(gx) + fabsf(gy) + fabsf(gz);
}

/* Backward (C) occupancy: neighbours count when their screen point lies in the
 * pixel (backward.cu:654-689). */
static float occ_mag_pix(const f2 *scr, int G, int g, int S, const float *cf, unsigned px, unsigned py) {
    int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G, off = (S - 1) / 2;
    float gx = 0.0f, gy = 0.0f, gz = 0.0f;
    for (int s = 0; s < S; s++) {
        int r = s - off, n;
        int ox = 0, oy = 0, oz = 0;
        n = x + r; if (n >= 0 && n < G && in_pixel(scr[z * G * G + y * G + n], px, py)) ox = 1;
        gx += cf[s] * (float)ox;
        n = y + r; if (n >= 0 && n < G && in_pixel(scr[z * G * G + n * G + x], px, py)) oy = 1;
        gy += cf[s] * (float)oy;
        n = z + r; if (n >= 0 && n < G && in_pixel(scr[n * G * G + y * G + x], px, py)) oz = 1;
        gz += cf[s] * (float)oz;
    }
    return fabsf(gx) + fabsf(gy) + fabsf(gz);
}

static float sigm(float x) { return 1.0f / (1.0f + expf(-x)); }

/* Test helper for the exact-gradient mode: the grid points of primitive q that
 * form its record at pixel (px, py) in the forward (forward projection, conf > 0,
 * stencil magnitude > 1e-7; forward.cu:481-627) and their magnitudes.  Returns
 * their count; lanes/mags hold at least G^3 entries.  Not part of the reference. */
int vio_record_lanes(const vio_params *p, uint32_t q, unsigned px, unsigned py, int32_t *lanes, float *mags) {
    int G = p->G, V = G * G * G, S, n = 0;
    float cf[5];
    stencil(p->genus, &S, cf);
    f3 c = {p->means[3 * q], p->means[3 * q + 1], p->means[3 * q + 2]};
    float step = G > 1 ? p->scale / (float)(G - 1) : p->scale;
    float gof = (float)(G - 1) / 2.0f;
    const float *conf = p->conf + (uint64_t)q * V;
    for (int g = 0; g < V; g++) {
        if (!(conf[g] > 0.0f)) continue;
        int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G;
        float rx = ((float)x - gof) * step, ry = ((float)y - gof) * step, rz = ((float)z - gof) * step;
        f3 pos = {c.x + rx, c.y + ry, c.z + rz};
        float h[4];
        t44(pos, p->proj, h);
        float pw = 1.0f / (h[3] + 0.0000001f);
        f2 s = {ndc2pix(h[0] * pw, p->W), ndc2pix(h[1] * pw, p->H)};
        if (!in_pixel(s, px, py)) continue;
        float m = occ_mag_conf(conf, G, g, S, cf);
        if (m > 1e-7f) {
            lanes[n] = g;
            mags[n] = m;
            n++;
        }
    }
    return n;
}

/* ------------------------------------------------------------------------ */
/* R5: render (forward.cu:146-792), per tile, program order                   */
/* ------------------------------------------------------------------------ */
/* skips (optional, per pixel): entries an active pixel visited while not done
 * that no grid point covers (occupancy sum < 1e-7).  At exactly these events
 * the reference kernel's thread leaves the loop body before the CTA barrier at
 * forward.cu:715 (forward.cu:629-631), so a scene with zero skips is one on
 * which every reference thread takes every barrier. */
void vio_render(const vio_params *p, const uint32_t *ranges, const uint32_t *point_list,
                const uint8_t *tile_mask, int nthreads,
                float *out_color, float *out_feat, float *vis,
                float *final_T, int32_t *n_contrib, int32_t *contrib_idx, float *delta_t, int32_t *skips) {
    int W = p->W, H = p->H, G = p->G, V = G * G * G, D = p->L * p->F, O = 3 + p->Fout + 1;
    int K = p->K;
    unsigned gxn = (W + TILE - 1) / TILE, gyn = (H + TILE - 1) / TILE;
    int S;
    float cf[5];
    stencil(p->genus, &S, cf);
    long ntiles = (long)gxn * gyn;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel
#endif
    {
        float *conf = malloc(sizeof(float) * V), *phi = malloc(sizeof(float) * V * (D > 0 ? D : 1));
        float *mlp = malloc(sizeof(float) * V * O);
        f2 *scr = malloc(sizeof(f2) * V);
        float *mag = malloc(sizeof(float) * V);
        /* per-pixel state */
        float T[256], C[256][3], *Fe = malloc(sizeof(float) * 256 * (p->Fout + 1));
        int cnt[256], done[256], has_p[256];
        float *pend = malloc(sizeof(float) * 256 * O);
        float pend_depth[256], T_pend[256];
        uint32_t pend_idx[256];
        float *acc = malloc(sizeof(float) * O);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (long t = 0; t < ntiles; t++) {
            if (tile_mask && !tile_mask[t]) continue;
            unsigned bx = t % gxn, by = t / gxn;
            for (int k = 0; k < 256; k++) {
                unsigned px = bx * TILE + k % TILE, py = by * TILE + k / TILE;
                T[k] = 1.0f; C[k][0] = C[k][1] = C[k][2] = 0.0f;
                for (int f = 0; f < p->Fout; f++) Fe[k * (p->Fout + 1) + f] = 0.0f;
                cnt[k] = 0; has_p[k] = 0; done[k] = !(px < (unsigned)W && py < (unsigned)H);
                pend_depth[k] = p->near_plane; T_pend[k] = 0.0f; pend_idx[k] = 0;
            }
            uint32_t r0 = ranges[2 * t], r1 = ranges[2 * t + 1];
            for (uint32_t j = r0; j < r1; j++) {
                int any = 0;
                for (int k = 0; k < 256; k++) any |= !done[k];
                if (!any) break; /* all pixels done: nothing further changes */
                uint32_t q = point_list[j];
                stage1(p, q, 1, conf, scr, phi, mlp);
                for (int g = 0; g < V; g++) mag[g] = occ_mag_conf(conf, G, g, S, cf);
                f3 c = {p->means[3 * q], p->means[3 * q + 1], p->means[3 * q + 2]};
                float depth = t43(c, p->view).z;
                for (int k = 0; k < 256; k++) {
                    if (done[k]) continue;
                    unsigned px = bx * TILE + k % TILE, py = by * TILE + k / TILE;
                    for (int o = 0; o < O; o++) acc[o] = 0.0f;
                    float ogs = 0.0f;
                    for (int g = 0; g < V; g++) {
                        if (!in_pixel(scr[g], px, py) || conf[g] <= 0.0f) continue;
                        float m = mag[g];
                        ogs += m;
                        if (m > 1e-7f) {
                            float w = conf[g] * m;
                            for (int o = 0; o < O; o++) acc[o] += mlp[(size_t)g * O + o] * w;
                        }
                    }
                    if (ogs < 1e-7f) {
                        if (skips) skips[(size_t)py * W + px]++;
                        continue;
                    }
                    for (int o = 0; o < O; o++) {
                        acc[o] += p->bl[o];
                        acc[o] = o < O - 1 ? sigm(acc[o]) : expf(acc[o]);
                    }
                    float *pp = pend + (size_t)k * O;
                    float *fe = Fe + k * (p->Fout + 1);
                    if (has_p[k]) {
                        float dt = fmaxf(0.0f, depth - pend_depth[k]);
                        if (dt > 1e-5f && cnt[k] < K) {
                            float alpha = 1.0f - expf(-pp[O - 1] * dt);
                            alpha = fminf(fmaxf(alpha, 0.0f), 1.0f);
                            float wgt = T_pend[k] * alpha;
                            for (int ch = 0; ch < 3; ch++) C[k][ch] += wgt * pp[ch];
                            for (int f = 0; f < p->Fout; f++) fe[f] += wgt * pp[3 + f];
                            T[k] = T_pend[k] * (1.0f - alpha);
                            size_t pix = (size_t)py * W + px;
                            contrib_idx[pix * K + cnt[k]] = (int32_t)pend_idx[k];
                            delta_t[pix * K + cnt[k]] = dt;
                            cnt[k]++;
                        }
                    }
                    if (T[k] >= 1e-4f && cnt[k] < K) {
                        for (int o = 0; o < O; o++) pp[o] = acc[o];
                        pend_depth[k] = depth; pend_idx[k] = j; has_p[k] = 1; T_pend[k] = T[k];
                    } else { has_p[k] = 0; done[k] = 1; }
                    if (T[k] < 1e-4f || cnt[k] >= K) done[k] = 1;
                }
            }
            for (int k = 0; k < 256; k++) {
                unsigned px = bx * TILE + k % TILE, py = by * TILE + k / TILE;
                if (!(px < (unsigned)W && py < (unsigned)H)) continue;
                size_t pix = (size_t)py * W + px;
                float *pp = pend + (size_t)k * O;
                float *fe = Fe + k * (p->Fout + 1);
                if (has_p[k] && T[k] >= 1e-4f && cnt[k] < K) {
                    float dt = fmaxf(0.0f, p->max_distance - pend_depth[k]);
                    if (dt > 1e-5f) {
                        float alpha = 1.0f - expf(-pp[O - 1] * dt);
                        alpha = fminf(fmaxf(alpha, 0.0f), 1.0f);
                        float wgt = T_pend[k] * alpha;
                        for (int ch = 0; ch < 3; ch++) C[k][ch] += wgt * pp[ch];
                        for (int f = 0; f < p->Fout; f++) fe[f] += wgt * pp[3 + f];
                        T[k] = T_pend[k] * (1.0f - alpha);
                        contrib_idx[pix * K + cnt[k]] = (int32_t)pend_idx[k];
                        delta_t[pix * K + cnt[k]] = dt;
                        cnt[k]++;
                    }
                }
                for (int ch = 0; ch < 3; ch++) {
                    float v = C[k][ch] + T[k] * p->bg[ch];
                    out_color[(size_t)ch * H * W + pix] = fminf(fmaxf(v, 0.0f), 1.0f);
                }
                for (int f = 0; f < p->Fout; f++) out_feat[(size_t)f * H * W + pix] = fe[f];
                vis[pix] = 1.0f - T[k];
                final_T[pix] = T[k];
                n_contrib[pix] = cnt[k];
            }
        }
        free(conf); free(phi); free(mlp); free(scr); free(mag); free(Fe); free(pend); free(acc);
    }
}

/* ------------------------------------------------------------------------ */
/* R7: backward (backward.cu:51-792), per tile, reverse list order            */
/* ------------------------------------------------------------------------ */
void vio_backward(const vio_params *p, const uint32_t *ranges, const uint32_t *point_list, uint64_t R,
                  const uint8_t *tile_mask, int nthreads,
                  const float *dL_dcolor, const float *dL_dfeat,
                  const int32_t *n_contrib, const int32_t *contrib_idx, const float *delta_t,
                  float *dconf, float *dtable, float *dW, float *db) {
    int W = p->W, H = p->H, G = p->G, V = G * G * G, D = p->L * p->F, O = 3 + p->Fout + 1;
    int K = p->K, B = O - 1;
    unsigned gxn = (W + TILE - 1) / TILE, gyn = (H + TILE - 1) / TILE;
    int S;
    float cf[5];
    stencil(p->genus, &S, cf);
    long ntiles = (long)gxn * gyn;
    int threaded = 0;
#ifdef _OPENMP
    if (nthreads > 0) omp_set_num_threads(nthreads);
    threaded = nthreads != 1;
#pragma omp parallel
#endif
    {
        float *conf = malloc(sizeof(float) * V), *phi = malloc(sizeof(float) * V * (D > 0 ? D : 1));
        float *mlp = malloc(sizeof(float) * V * O);
        f2 *scr = malloc(sizeof(f2) * V);
        float *mag = malloc(sizeof(float) * V);
        float *dOut = malloc(sizeof(float) * 256 * B), *after = malloc(sizeof(float) * 256 * B);
        int next[256];
        float *in = malloc(sizeof(float) * (D > 0 ? D : 1)), *agg = malloc(sizeof(float) * O);
        float *blend = malloc(sizeof(float) * B), *dpre = malloc(sizeof(float) * O);
        float *dIn = malloc(sizeof(float) * (D > 0 ? D : 1)), *dphi = malloc(sizeof(float) * (p->F > 0 ? p->F : 1));
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 4)
#endif
        for (long t = 0; t < ntiles; t++) {
            if (tile_mask && !tile_mask[t]) continue;
            unsigned bx = t % gxn, by = t / gxn;
            for (int k = 0; k < 256; k++) {
                unsigned px = bx * TILE + k % TILE, py = by * TILE + k / TILE;
                next[k] = -1;
                if (px < (unsigned)W && py < (unsigned)H) {
                    size_t pix = (size_t)py * W + px;
                    int nc = n_contrib[pix] < K ? n_contrib[pix] : K;
                    next[k] = nc - 1;
                    for (int c = 0; c < 3; c++) { dOut[k * B + c] = dL_dcolor[(size_t)c * H * W + pix]; after[k * B + c] = p->bg[c]; }
                    for (int f = 0; f < p->Fout; f++) {
                        dOut[k * B + 3 + f] = dL_dfeat ? dL_dfeat[(size_t)f * H * W + pix] : 0.0f;
                        after[k * B + 3 + f] = 0.0f;
                    }
                }
            }
            uint32_t r0 = ranges[2 * t], r1 = ranges[2 * t + 1];
            for (int64_t j = (int64_t)r1 - 1; j >= (int64_t)r0; j--) {
                uint32_t q = point_list[j];
                if (q >= (uint32_t)p->P) continue;
                int need = 0;
                for (int k = 0; k < 256; k++) need |= next[k] >= 0;
                if (!need) break; /* no pixel expects anything: no further effect */
                stage1(p, q, 0, conf, scr, phi, mlp);
                for (int g = 0; g < V; g++) mag[g] = occ_mag_conf(conf, G, g, S, cf);
                f3 c = {p->means[3 * q], p->means[3 * q + 1], p->means[3 * q + 2]};
                float step = G > 1 ? p->scale / (float)(G - 1) : p->scale;
                float gof = (float)(G - 1) / 2.0f;
                for (int k = 0; k < 256; k++) {
                    if (next[k] < 0) continue;
                    unsigned px = bx * TILE + k % TILE, py = by * TILE + k / TILE;
                    size_t pix = (size_t)py * W + px;
                    uint32_t stored = (uint32_t)contrib_idx[pix * K + next[k]];
                    uint32_t expect = stored < R ? point_list[stored] : 0xFFFFFFFFu;
                    if (q != expect) continue;
                    float dt = delta_t[pix * K + next[k]];
                    for (int i = 0; i < D; i++) in[i] = 0.0f;
                    for (int o = 0; o < O; o++) agg[o] = 0.0f;
                    for (int g = 0; g < V; g++) {
                        if (!in_pixel(scr[g], px, py) || conf[g] <= 0.0f) continue;
                        float m = mag[g];
                        if (m > 1e-7f) {
                            float w = conf[g] * m;
                            for (int i = 0; i < D; i++) in[i] += phi[(size_t)g * D + i] * w;
                            for (int o = 0; o < O; o++) agg[o] += mlp[(size_t)g * O + o] * w;
                        }
                    }
                    float dens = 0.0f;
                    for (int o = 0; o < O; o++) {
                        float pre = agg[o] + p->bl[o];
                        if (o < B) blend[o] = 1.0f / (1.0f + expf(-pre));
                        else dens = expf(pre);
                    }
                    float *dO = dOut + k * B, *af = after + k * B;
                    float dalpha = 0.0f;
                    for (int d = 0; d < B; d++) { float dbl = dO[d] * blend[d]; dalpha += dbl * (blend[d] - af[d]); }
                    for (int d = 0; d < B; d++) { float y = blend[d]; dpre[d] = dO[d] * blend[d] * y * (1.0f - y); }
                    dpre[O - 1] = dalpha * dens * dt * dens;
                    for (int jj = 0; jj < D; jj++) {
                        float s = 0.0f;
                        for (int o = 0; o < O; o++) s += dpre[o] * p->Wl[o * D + jj];
                        dIn[jj] = s;
                    }
                    for (int o = 0; o < O; o++) {
                        if (threaded) {
#pragma omp atomic
                            db[o] += dpre[o];
                        } else db[o] += dpre[o];
                        for (int i = 0; i < D; i++) {
                            float v = dpre[o] * in[i];
                            if (threaded) {
#pragma omp atomic
                                dW[o * D + i] += v;
                            } else dW[o * D + i] += v;
                        }
                    }
                    for (int g = 0; g < V; g++) {
                        float m2 = occ_mag_pix(scr, G, g, S, cf, px, py);
                        if (!(m2 > 1e-7f)) continue;
                        float dX = 0.0f;
                        for (int f = 0; f < D; f++) dX += dIn[f] * phi[(size_t)g * D + f];
                        dX *= m2;
                        if (threaded) {
#pragma omp atomic
                            dconf[(uint64_t)q * V + g] += dX;
                        } else dconf[(uint64_t)q * V + g] += dX;
                        float wg = m2 * conf[g];
                        if (!(fabsf(wg) > 1e-9f)) continue;
                        int z = g / (G * G), rem = g % (G * G), y = rem / G, x = rem % G;
                        f3 pos = {c.x + ((float)x - gof) * step, c.y + ((float)y - gof) * step, c.z + ((float)z - gof) * step};
                        for (int l = 0; l < p->L; l++) {
                            for (int f = 0; f < p->F; f++) dphi[f] = dIn[l * p->F + f] * wg;
                            hash_grad(p, pos, l, dphi, dtable, threaded);
                        }
                    }
                    for (int d = 0; d < B; d++) {
                        dO[d] *= blend[d];
                        af[d] = blend[d] + af[d] * (1.0f - blend[d]);
                    }
                    next[k]--;
                }
            }
        }
        free(conf); free(phi); free(mlp); free(scr); free(mag); free(dOut); free(after);
        free(in); free(agg); free(blend); free(dpre); free(dIn); free(dphi);
    }
}
