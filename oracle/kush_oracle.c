/*
 * kush_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C restatement of kushkash's CPU kernels (kushkash/kush/cpu.mojo) and of the shared cache format
 * (kushkash/kush/quant.mojo), used only as the parity checker for the sm_100a CUDA library and as the timed
 * CPU baseline in bench.py.  Nothing in the product path (kushkash_b200/) may load or call this library.
 *
 * Why a restatement: the reference's own CPU library (libkush_cpu.so) is built from Mojo sources by the
 * `mojo` compiler, which is not installed here (and there is no network), so it cannot be compiled or run.
 * This file follows the Mojo code step by step; every function cites the file:line it restates.  It is pinned
 * against the reference's own PyTorch pins (tests/test_cpu.py:16-24 ref_quantize, kushkash/_ops.py
 * dequant_records / cached_kv / unpack_reference / fwht_reference) through the fixtures in tests/golden/.
 *
 * C ABI: the five entry points of kushkash/_cpu.py:10-40 with the same argument lists (every integer and
 * address is int64, the softmax scale is float; return 0, or -1 for an unsupported head_dim / bits), all with
 * the reference's 32-token page.  The `_p` variants take the page size P (16 or 32) as an extra first argument;
 * kushkash's own format is P = 32 (quant.mojo:16), P = 16 is the same layout with 16 token rows.
 *
 * Arithmetic: fp32 throughout, IEEE division, round-half-to-even codes (torch.round, as the reference's tests
 * pin), fp16 scale/bias rounding to nearest even.  Build with -ffp-contract=off and without -ffast-math.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------ fp16 <-> fp32 */
/* IEEE binary16 <-> binary32, round to nearest even (what Mojo's .cast[DType.float16]() and torch .half() do). */
static float h2f(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, x;
    if (e == 0) {
        if (m == 0) {
            x = sign;
        } else {                                   /* subnormal: renormalise */
            e = 113;
            while (!(m & 0x400)) { m <<= 1; e--; }
            x = sign | (e << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) {
        x = sign | 0x7f800000 | (m << 13);
    } else {
        x = sign | ((e + 112) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &x, 4);
    return f;
}

static uint16_t f2h(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint16_t sign = (uint16_t)((x >> 16) & 0x8000);
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u)                         /* inf / nan */
        return sign | 0x7c00 | (ax > 0x7f800000u ? (0x200 | ((ax >> 13) & 0x3ff)) : 0);
    if (ax >= 0x477ff000u)                         /* >= 65520 rounds to inf */
        return sign | 0x7c00;
    if (ax < 0x38800000u) {                        /* below 2^-14: subnormal half (or zero) */
        uint32_t e = ax >> 23;
        if (e < 102) return sign;                  /* below 2^-25: rounds to zero */
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        uint32_t shift = 126 - e;                  /* value / 2^-24 = m >> shift */
        uint32_t q = m >> shift, rem = m & ((1u << shift) - 1), halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (q & 1))) q++;
        return sign | (uint16_t)q;
    }
    uint32_t hbits = (ax >> 13) - (112u << 10);
    uint32_t rem = ax & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (hbits & 1))) hbits++;
    return sign | (uint16_t)hbits;
}

/* exported for the oracle's own tests (checked against numpy.float16) */
float kush_oracle_h2f(uint16_t h) { return h2f(h); }
uint16_t kush_oracle_f2h(float f) { return f2h(f); }

/* ------------------------------------------------------------------ format (quant.mojo:19-87) */
typedef struct {
    int D, bits, P;
    int DC;                                        /* bytes per token row: D (int8) or D/2 (int4), quant.mojo:20-22 */
    int rb, off_vq, off_ks, off_kb, off_vs, off_vb; /* record layout, quant.mojo:53-87 */
} fmt_t;

static int fmt_init(fmt_t *f, int64_t D, int64_t bits, int64_t P) {
    if (!(D == 64 || D == 128 || D == 256) || !(bits == 4 || bits == 8) || !(P == 16 || P == 32)) return -1;
    f->D = (int)D; f->bits = (int)bits; f->P = (int)P;
    f->DC = bits == 8 ? f->D : f->D / 2;
    f->off_vq = f->P * f->DC;
    f->off_ks = 2 * f->P * f->DC;
    f->off_kb = f->off_ks + 2 * f->D;
    f->off_vs = f->off_ks + 4 * f->D;
    f->off_vb = f->off_vs + 2 * f->P;
    f->rb = 2 * f->P * f->DC + 4 * f->D + 4 * f->P;
    return 0;
}

/* quant.mojo:25-35 qparams: scale and bias rounded to fp16, codes computed against the rounded values */
static void qparams(int bits, float mn, float mx, float *s, float *b, float *inv) {
    const float levels = (float)((1 << bits) - 1), halfv = (float)(1 << (bits - 1));
    float sc = h2f(f2h((mx - mn) / levels));
    float prod = sc * halfv;                       /* exact: power-of-two multiply */
    float bi = h2f(f2h(mn + prod));
    *s = sc;
    *b = bi;
    *inv = sc > 0.0f ? 1.0f / sc : 0.0f;
}

/* quant.mojo:38-44 qcode: round((x - b) * inv), clamp to [-HALF, HALF - 1]; ties to even */
static int8_t qcode(int bits, float x, float b, float inv) {
    const float halfv = (float)(1 << (bits - 1));
    float d = x - b;
    float r = nearbyintf(d * inv);
    if (r < -halfv) r = -halfv;
    if (r > halfv - 1.0f) r = halfv - 1.0f;
    return (int8_t)r;
}

/* quant.mojo:47-50 pack4: lo in bits 0-3, hi in bits 4-7 */
static uint8_t pack4(int8_t lo, int8_t hi) { return (uint8_t)(((uint8_t)lo & 0x0f) | ((uint8_t)hi << 4)); }

static void store_h(uint8_t *p, int i, float v) {
    uint16_t h = f2h(v);
    memcpy(p + 2 * i, &h, 2);
}

static float load_h(const uint8_t *p, int i) {
    uint16_t h;
    memcpy(&h, p + 2 * i, 2);
    return h2f(h);
}

/* ------------------------------------------------------------------ cache addressing (cpu.mojo:48-71) */
typedef struct {
    uint8_t *cache;
    int64_t bs, hs;                                /* byte strides of (block, kv head) */
    float *tail_k;                                 /* [slots][H][P][D] fp32 */
    const int32_t *tail_idx, *block_table;
    int64_t max_pages;                             /* block_table row stride (elements) */
    int64_t hkv;
} cache_t;

static uint8_t *rec_of(const cache_t *c, int64_t s, int64_t lp, int64_t h) {
    int64_t blk = c->block_table[s * c->max_pages + lp];
    return c->cache + blk * c->bs + h * c->hs;
}

static int64_t tail_off(const cache_t *c, const fmt_t *f, int64_t s, int64_t h) {
    return ((int64_t)c->tail_idx[s] * c->hkv + h) * f->P * f->D;   /* element offset of the tail page */
}

/* ------------------------------------------------------------------ write path */
/* cpu.mojo:173-218 _quantize_k_page: per-channel range over the page's P tokens; row t < split from the tail
 * (ka + t*sa), the rest from this step's rows (kb_src + (t - split)*skb) */
static void quantize_k_page(const fmt_t *f, const float *ka, int64_t sa, const float *kb_src, int64_t skb,
                            int split, uint8_t *rec) {
    const int D = f->D, P = f->P, DC = f->DC;
    float bias[256], inv[256];
    for (int d = 0; d < D; d++) {
        float mn = INFINITY, mx = -INFINITY;
        for (int t = 0; t < P; t++) {
            float x = t < split ? ka[t * sa + d] : kb_src[(t - split) * skb + d];
            mn = fminf(mn, x);
            mx = fmaxf(mx, x);
        }
        float s, b, iv;
        qparams(f->bits, mn, mx, &s, &b, &iv);
        store_h(rec + f->off_ks, d, s);
        store_h(rec + f->off_kb, d, b);
        bias[d] = b;
        inv[d] = iv;
    }
    for (int t = 0; t < P; t++) {
        const float *row = t < split ? ka + t * sa : kb_src + (t - split) * skb;
        uint8_t *kc = rec + (int64_t)t * DC;
        if (f->bits == 8) {
            for (int d = 0; d < D; d++) kc[d] = (uint8_t)qcode(8, row[d], bias[d], inv[d]);
        } else {
            for (int j = 0; j < D / 2; j++)
                kc[j] = pack4(qcode(4, row[j], bias[j], inv[j]), qcode(4, row[j + D / 2], bias[j + D / 2], inv[j + D / 2]));
        }
    }
}

/* cpu.mojo:221-245 _quantize_v_row: per-token range over the D channels; the row's final encoding */
static void quantize_v_row(const fmt_t *f, const float *row, uint8_t *rec, int t) {
    const int D = f->D;
    float mn = INFINITY, mx = -INFINITY;
    for (int d = 0; d < D; d++) {
        mn = fminf(mn, row[d]);
        mx = fmaxf(mx, row[d]);
    }
    float s, b, iv;
    qparams(f->bits, mn, mx, &s, &b, &iv);
    store_h(rec + f->off_vs, t, s);
    store_h(rec + f->off_vb, t, b);
    uint8_t *vc = rec + f->off_vq + (int64_t)t * f->DC;
    if (f->bits == 8) {
        for (int d = 0; d < D; d++) vc[d] = (uint8_t)qcode(8, row[d], b, iv);
    } else {
        for (int j = 0; j < D / 2; j++) vc[j] = pack4(qcode(4, row[j], b, iv), qcode(4, row[j + D / 2], b, iv));
    }
}

/* cpu.mojo:248-270 _append (GPU twin gpu.mojo:207-238): one token per sequence at pos = seq_lens[s] + pos_offset;
 * negative positions (padding rows) are skipped; K to the exact tail, V quantized into record row `slot`; the
 * last slot of a page quantizes the page's K from the tail; advance stores pos + 1 */
static void do_append(const fmt_t *f, const float *k_new, const float *v_new, int64_t ks, int64_t vs, int32_t *seq_lens,
                      int64_t pos_offset, int advance, const cache_t *c, int64_t S) {
    const int D = f->D, P = f->P;
    for (int64_t s = 0; s < S; s++) {
        int64_t pos = (int64_t)seq_lens[s] + pos_offset;
        if (pos < 0) continue;
        int slot = (int)(pos % P);
        for (int64_t h = 0; h < c->hkv; h++) {
            float *tk = c->tail_k + tail_off(c, f, s, h);
            memcpy(tk + (int64_t)slot * D, k_new + s * ks + h * D, sizeof(float) * D);
            uint8_t *rec = rec_of(c, s, pos / P, h);
            quantize_v_row(f, v_new + s * vs + h * D, rec, slot);
            if (slot == P - 1) quantize_k_page(f, tk, D, tk, D, P, rec);
        }
        if (advance) seq_lens[s] = (int32_t)(pos + 1);
    }
}

/* cpu.mojo:273-304 _write (GPU twin gpu.mojo:241-276): sequence s owns rows [qsl[s], qsl[s+1]) at positions
 * [ctx, seq_lens[s]); job j covers logical page job_page[j] of job_seq[j].  mode 0: V rows of the page, and K of
 * the page if it is now complete (older rows from the tail, newer from the new rows).  mode 1: for a page still
 * partial, copy its new K rows into the tail. */
static void do_write(const fmt_t *f, const float *k_new, const float *v_new, int64_t ks, int64_t vs, const int32_t *qsl,
                     const int32_t *seq_lens, const int32_t *job_seq, const int32_t *job_page, int64_t n_jobs, int64_t mode,
                     const cache_t *c) {
    const int D = f->D, P = f->P;
    for (int64_t j = 0; j < n_jobs; j++) {
        int64_t s = job_seq[j];
        int64_t ps = (int64_t)job_page[j] * P;
        int64_t q0 = qsl[s];
        int64_t total = seq_lens[s];
        int64_t ctx = total - ((int64_t)qsl[s + 1] - q0);
        int complete = ps + P <= total;
        if (mode != 0 && complete) continue;
        for (int64_t h = 0; h < c->hkv; h++) {
            float *tb = c->tail_k + tail_off(c, f, s, h);
            if (mode == 0) {
                uint8_t *rec = rec_of(c, s, ps / P, h);
                int64_t t0 = ps > ctx ? ps : ctx, t1 = ps + P < total ? ps + P : total;
                for (int64_t t = t0; t < t1; t++) quantize_v_row(f, v_new + (q0 + t - ctx) * vs + h * D, rec, (int)(t - ps));
                if (complete) {
                    int64_t split = ctx - ps;
                    if (split > P) split = P;
                    if (split < 0) split = 0;
                    quantize_k_page(f, tb, D, k_new + (q0 + ps + split - ctx) * ks + h * D, ks, (int)split, rec);
                }
            } else {
                for (int64_t t = ps > ctx ? ps : ctx; t < total; t++)
                    memcpy(tb + (t - ps) * D, k_new + (q0 + t - ctx) * ks + h * D, sizeof(float) * D);
            }
        }
    }
}

/* ------------------------------------------------------------------ decode */
/* cpu.mojo:309-317 _codes: code of dim d of a token row as fp32 (int4: dim d < D/2 low nibble of byte d, else the
 * high nibble of byte d - D/2; two's complement) */
static void unpack_row(const fmt_t *f, const uint8_t *row, float *out) {
    const int D = f->D;
    if (f->bits == 8) {
        for (int d = 0; d < D; d++) out[d] = (float)(int8_t)row[d];
    } else {
        for (int j = 0; j < D / 2; j++) {
            int8_t b = (int8_t)row[j];
            out[j] = (float)(int8_t)((int8_t)(b << 4) >> 4);
            out[j + D / 2] = (float)(int8_t)(b >> 4);
        }
    }
}

/* page-granular online-softmax step over the cnt scores of head g (cpu.mojo:352-368) */
static float softmax_page(float *row, int cnt, float *m, float *l) {
    float pm = -INFINITY;
    for (int t = 0; t < cnt; t++) pm = fmaxf(pm, row[t]);
    float mo = *m, mn = fmaxf(mo, pm);
    float corr = expf(mo - mn);
    float tot = 0.0f;
    for (int t = 0; t < cnt; t++) {
        float e = expf(row[t] - mn);
        row[t] = e;
        tot += e;
    }
    *m = mn;
    *l = *l * corr + tot;
    return corr;
}

/* cpu.mojo:320-451 _decode_task: attention of the G q heads of (sequence s, kv head h) over its whole cache.
 * Per full page the K scale folds into q and the K bias into one scalar per head; V scales fold into the
 * softmax weights and V biases into one scalar per head.  The partial last page takes K from the exact tail. */
static void decode_task(const fmt_t *f, const float *q, float *o, const cache_t *c, const int32_t *seq_lens, int G,
                        float sm, int64_t s, int64_t h, float *scr) {
    const int D = f->D, P = f->P, DC = f->DC;
    const int64_t H = c->hkv;
    int64_t n = seq_lens[s];
    int64_t qb = (s * H + h) * G * D;
    float *qsm = scr, *qs = qsm + G * D, *acc = qs + G * D, *crow = acc + G * D, *sc = crow + D;
    float *m = sc + G * P, *l = m + G, *vbacc = l + G, *kbs = vbacc + G;
    for (int g = 0; g < G; g++) {
        for (int d = 0; d < D; d++) {
            qsm[g * D + d] = q[qb + g * D + d] * sm;
            acc[g * D + d] = 0.0f;
        }
        m[g] = -INFINITY;
        l[g] = 0.0f;
        vbacc[g] = 0.0f;
    }
    for (int64_t lp = 0; lp < n / P; lp++) {
        const uint8_t *rec = rec_of(c, s, lp, h);
        for (int g = 0; g < G; g++) {
            float kbias = 0.0f;
            for (int d = 0; d < D; d++) {
                float qv = qsm[g * D + d];
                qs[g * D + d] = qv * load_h(rec + f->off_ks, d);
                kbias += qv * load_h(rec + f->off_kb, d);
            }
            kbs[g] = kbias;
        }
        for (int t = 0; t < P; t++) {
            unpack_row(f, rec + (int64_t)t * DC, crow);
            for (int g = 0; g < G; g++) {
                float dot = 0.0f;
                for (int d = 0; d < D; d++) dot += qs[g * D + d] * crow[d];
                sc[g * P + t] = dot + kbs[g];
            }
        }
        for (int g = 0; g < G; g++) {
            float corr = softmax_page(sc + g * P, P, m + g, l + g);
            vbacc[g] *= corr;
            for (int d = 0; d < D; d++) acc[g * D + d] *= corr;
        }
        for (int t = 0; t < P; t++) {
            unpack_row(f, rec + f->off_vq + (int64_t)t * DC, crow);
            float vst = load_h(rec + f->off_vs, t), vbt = load_h(rec + f->off_vb, t);
            for (int g = 0; g < G; g++) {
                float e = sc[g * P + t];
                vbacc[g] += e * vbt;
                float wv = e * vst;
                for (int d = 0; d < D; d++) acc[g * D + d] += wv * crow[d];
            }
        }
    }
    int tail_n = (int)(n % P);
    if (tail_n > 0) {                              /* cpu.mojo:418-444 */
        const float *tk = c->tail_k + tail_off(c, f, s, h);
        const uint8_t *vrec = rec_of(c, s, n / P, h);
        for (int g = 0; g < G; g++) {
            for (int t = 0; t < tail_n; t++) {
                float dot = 0.0f;
                for (int d = 0; d < D; d++) dot += qsm[g * D + d] * tk[t * D + d];
                sc[g * P + t] = dot;
            }
            float corr = softmax_page(sc + g * P, tail_n, m + g, l + g);
            vbacc[g] *= corr;
            for (int d = 0; d < D; d++) acc[g * D + d] *= corr;
        }
        for (int t = 0; t < tail_n; t++) {
            unpack_row(f, vrec + f->off_vq + (int64_t)t * DC, crow);
            float vst = load_h(vrec + f->off_vs, t), vbt = load_h(vrec + f->off_vb, t);
            for (int g = 0; g < G; g++) {
                float e = sc[g * P + t];
                vbacc[g] += e * vbt;
                float wv = e * vst;
                for (int d = 0; d < D; d++) acc[g * D + d] += wv * crow[d];
            }
        }
    }
    for (int g = 0; g < G; g++) {                  /* cpu.mojo:446-450 */
        float inv_l = l[g] > 0.0f ? 1.0f / l[g] : 0.0f;
        for (int d = 0; d < D; d++) o[qb + g * D + d] = (acc[g * D + d] + vbacc[g]) * inv_l;
    }
}

static int g_threads = 0;                          /* 0: OpenMP default */

/* thread count for the decode task pool (bench.py's CPU baseline records it); returns the count in use */
int kush_oracle_set_threads(int64_t n) {
    g_threads = (int)n;
#ifdef _OPENMP
    return n > 0 ? (int)n : omp_get_max_threads();
#else
    return 1;
#endif
}

/* cpu.mojo:454-466 _decode: one task per (sequence, kv head); below ~256 pages of work the tasks run inline */
static void do_decode(const fmt_t *f, const float *q, float *o, const cache_t *c, const int32_t *seq_lens, int G, float sm,
                      int64_t S) {
    const int64_t H = c->hkv, tasks = S * H;
    const size_t nscr = (size_t)G * f->D * 3 + f->D + (size_t)G * (f->P + 4);
    int64_t pages = 0;
    for (int64_t s = 0; s < S; s++) pages += seq_lens[s] / f->P + 1;
    if (pages * H < 256) {
        float *scr = (float *)malloc(sizeof(float) * nscr);
        for (int64_t i = 0; i < tasks; i++) decode_task(f, q, o, c, seq_lens, G, sm, i / H, i % H, scr);
        free(scr);
        return;
    }
#ifdef _OPENMP
    int nt = g_threads > 0 ? g_threads : omp_get_max_threads();
#pragma omp parallel num_threads(nt)
#endif
    {
        float *scr = (float *)malloc(sizeof(float) * nscr);
#ifdef _OPENMP
#pragma omp for schedule(dynamic, 1)
#endif
        for (int64_t i = 0; i < tasks; i++) decode_task(f, q, o, c, seq_lens, G, sm, i / H, i % H, scr);
        free(scr);
    }
}

/* ------------------------------------------------------------------ rotation (quant.mojo:90-122, cpu.mojo:82-107) */
static const uint32_t FWHT_SCALE_BITS[3] = {0x3E000000u, 0x3DB504F3u, 0x3D800000u};   /* fp32 1/sqrt(D), D=64/128/256 */

/* canonical Walsh-Hadamard order: fp32 butterflies over strides 1, 2, ..., D/2 in that order, then one separate
 * multiply by fp32 1/sqrt(D) (no fusion into an FMA) */
static void fwht_rows(int D, float *x, int64_t rows) {
    uint32_t bits = FWHT_SCALE_BITS[D == 64 ? 0 : D == 128 ? 1 : 2];
    float sc;
    memcpy(&sc, &bits, 4);
    for (int64_t r = 0; r < rows; r++) {
        float *p = x + r * D;
        for (int h = 1; h < D; h <<= 1)
            for (int i = 0; i < D; i++)
                if (!(i & h)) {
                    float a = p[i], b = p[i + h];
                    p[i] = a + b;
                    p[i + h] = a - b;
                }
        for (int i = 0; i < D; i++) {
            volatile float y = p[i] * sc;          /* rounded on its own */
            p[i] = y;
        }
    }
}

/* ------------------------------------------------------------------ unpack (cpu.mojo:110-169) */
static float code_at(const fmt_t *f, const uint8_t *row, int c) {
    if (f->bits == 8) return (float)(int8_t)row[c];
    int8_t b = (int8_t)row[c % (f->D / 2)];
    return c < f->D / 2 ? (float)(int8_t)((int8_t)(b << 4) >> 4) : (float)(int8_t)(b >> 4);
}

/* history pages and partial pages dequantized with fma(code, scale, bias) in fp32, optionally rotated back, then
 * the new chunk's rows copied as they are */
static void do_unpack(const fmt_t *f, const uint8_t *cache, int64_t bs, int64_t hs, int64_t H, const int32_t *page_blk,
                      const int32_t *page_dst, int64_t n_pages, const int32_t *tail_blk, const int32_t *tail_info,
                      int64_t n_tail, const float *tail_k, const float *k_new, const float *v_new, int64_t ks_new,
                      int64_t vs_new, const int32_t *new_dst, int64_t n_new, float *kp, float *vp, int rot) {
    const int D = f->D, P = f->P, DC = f->DC;
    const int64_t rs = H * D;
    float kx[256], vx[256];
    for (int64_t b = 0; b < n_pages + n_tail; b++) {
        int page = b < n_pages;
        int64_t i = b - n_pages;
        int64_t blk = page ? page_blk[b] : tail_blk[i];
        int64_t dst0 = page ? page_dst[b] : tail_info[3 * i];
        int64_t n = page ? P : tail_info[3 * i + 1];
        for (int64_t h = 0; h < H; h++) {
            const uint8_t *rec = cache + blk * bs + h * hs;
            int64_t tk = page ? 0 : ((int64_t)tail_info[3 * i + 2] * H + h) * P * D;
            for (int64_t t = 0; t < n; t++) {
                float vs = load_h(rec + f->off_vs, (int)t), vb = load_h(rec + f->off_vb, (int)t);
                for (int cc = 0; cc < D; cc++) {
                    if (page)
                        kx[cc] = fmaf(code_at(f, rec + t * DC, cc), load_h(rec + f->off_ks, cc), load_h(rec + f->off_kb, cc));
                    else
                        kx[cc] = tail_k[tk + t * D + cc];
                    vx[cc] = fmaf(code_at(f, rec + f->off_vq + t * DC, cc), vs, vb);
                }
                if (rot) {
                    fwht_rows(D, kx, 1);
                    fwht_rows(D, vx, 1);
                }
                int64_t o = (dst0 + t) * rs + h * D;
                memcpy(kp + o, kx, sizeof(float) * D);
                memcpy(vp + o, vx, sizeof(float) * D);
            }
        }
    }
    for (int64_t j = 0; j < n_new; j++) {
        int64_t o = (int64_t)new_dst[j] * rs;
        for (int64_t h = 0; h < H; h++) {
            memcpy(kp + o + h * D, k_new + j * ks_new + h * D, sizeof(float) * D);
            memcpy(vp + o + h * D, v_new + j * vs_new + h * D, sizeof(float) * D);
        }
    }
}

/* ------------------------------------------------------------------ C ABI (kushkash/_cpu.py:10-40) */
#define I int64_t
#define PTR(T, a) ((T *)(intptr_t)(a))

static cache_t mk_cache(I cache, I bs, I hs, I tail_k, I tail_idx, I block_table, I max_pages, I hkv) {
    cache_t c = {PTR(uint8_t, cache), bs, hs, PTR(float, tail_k), PTR(const int32_t, tail_idx),
                 PTR(const int32_t, block_table), max_pages, hkv};
    return c;
}

int32_t kush_cpu_append_p(I page, I d, I bits, I k_new, I v_new, I k_stride, I v_stride, I seq_lens, I pos_offset,
                          I advance, I cache, I bs, I hs, I tail_k, I tail_idx, I block_table, I max_pages, I hkv,
                          I n_seqs) {
    fmt_t f;
    if (fmt_init(&f, d, bits, page)) return -1;
    cache_t c = mk_cache(cache, bs, hs, tail_k, tail_idx, block_table, max_pages, hkv);
    do_append(&f, PTR(const float, k_new), PTR(const float, v_new), k_stride, v_stride, PTR(int32_t, seq_lens),
              pos_offset, advance != 0, &c, n_seqs);
    return 0;
}

int32_t kush_cpu_write_p(I page, I d, I bits, I k_new, I v_new, I k_stride, I v_stride, I qsl, I seq_lens, I job_seq,
                         I job_page, I n_jobs, I mode, I cache, I bs, I hs, I tail_k, I tail_idx, I block_table,
                         I max_pages, I hkv) {
    fmt_t f;
    if (fmt_init(&f, d, bits, page)) return -1;
    cache_t c = mk_cache(cache, bs, hs, tail_k, tail_idx, block_table, max_pages, hkv);
    do_write(&f, PTR(const float, k_new), PTR(const float, v_new), k_stride, v_stride, PTR(const int32_t, qsl),
             PTR(const int32_t, seq_lens), PTR(const int32_t, job_seq), PTR(const int32_t, job_page), n_jobs, mode, &c);
    return 0;
}

int32_t kush_cpu_decode_p(I page, I d, I bits, I q, I o, I cache, I bs, I hs, I tail_k, I tail_idx, I block_table,
                          I seq_lens, I max_pages, I hkv, I group, float sm, I n_seqs) {
    fmt_t f;
    if (fmt_init(&f, d, bits, page) || group < 1) return -1;
    cache_t c = mk_cache(cache, bs, hs, tail_k, tail_idx, block_table, max_pages, hkv);
    do_decode(&f, PTR(const float, q), PTR(float, o), &c, PTR(const int32_t, seq_lens), (int)group, sm, n_seqs);
    return 0;
}

int32_t kush_cpu_unpack_p(I page, I d, I bits, I cache, I bs, I hs, I hkv, I page_blk, I page_dst, I n_pages, I tail_blk,
                          I tail_info, I n_tail, I tail_k, I k_new, I v_new, I k_stride, I v_stride, I new_dst, I n_new,
                          I kp, I vp, I rot) {
    fmt_t f;
    if (fmt_init(&f, d, bits, page)) return -1;
    do_unpack(&f, PTR(const uint8_t, cache), bs, hs, hkv, PTR(const int32_t, page_blk), PTR(const int32_t, page_dst),
              n_pages, PTR(const int32_t, tail_blk), PTR(const int32_t, tail_info), n_tail, PTR(const float, tail_k),
              PTR(const float, k_new), PTR(const float, v_new), k_stride, v_stride, PTR(const int32_t, new_dst), n_new,
              PTR(float, kp), PTR(float, vp), rot != 0);
    return 0;
}

/* the reference's exact entry points (page size 32) */
int32_t kush_cpu_append(I d, I bits, I k_new, I v_new, I k_stride, I v_stride, I seq_lens, I pos_offset, I advance,
                        I cache, I bs, I hs, I tail_k, I tail_idx, I block_table, I max_pages, I hkv, I n_seqs) {
    return kush_cpu_append_p(32, d, bits, k_new, v_new, k_stride, v_stride, seq_lens, pos_offset, advance, cache, bs, hs,
                             tail_k, tail_idx, block_table, max_pages, hkv, n_seqs);
}

int32_t kush_cpu_write(I d, I bits, I k_new, I v_new, I k_stride, I v_stride, I qsl, I seq_lens, I job_seq, I job_page,
                       I n_jobs, I mode, I cache, I bs, I hs, I tail_k, I tail_idx, I block_table, I max_pages, I hkv) {
    return kush_cpu_write_p(32, d, bits, k_new, v_new, k_stride, v_stride, qsl, seq_lens, job_seq, job_page, n_jobs, mode,
                            cache, bs, hs, tail_k, tail_idx, block_table, max_pages, hkv);
}

int32_t kush_cpu_decode(I d, I bits, I q, I o, I cache, I bs, I hs, I tail_k, I tail_idx, I block_table, I seq_lens,
                        I max_pages, I hkv, I group, float sm, I n_seqs) {
    return kush_cpu_decode_p(32, d, bits, q, o, cache, bs, hs, tail_k, tail_idx, block_table, seq_lens, max_pages, hkv,
                             group, sm, n_seqs);
}

int32_t kush_cpu_fwht(I d, I x, I rows) {
    if (!(d == 64 || d == 128 || d == 256)) return -1;
    fwht_rows((int)d, PTR(float, x), rows);
    return 0;
}

int32_t kush_cpu_unpack(I d, I bits, I cache, I bs, I hs, I hkv, I page_blk, I page_dst, I n_pages, I tail_blk,
                        I tail_info, I n_tail, I tail_k, I k_new, I v_new, I k_stride, I v_stride, I new_dst, I n_new,
                        I kp, I vp, I rot) {
    return kush_cpu_unpack_p(32, d, bits, cache, bs, hs, hkv, page_blk, page_dst, n_pages, tail_blk, tail_info, n_tail,
                             tail_k, k_new, v_new, k_stride, v_stride, new_dst, n_new, kp, vp, rot);
}
