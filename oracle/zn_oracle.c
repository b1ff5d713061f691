/*
 * CPU oracle for the cuZipNN codec path.  TEST INFRASTRUCTURE ONLY (see zn_oracle.h): it is
 * the checker for the CUDA library, never part of it.  Scalar, readable code; the only
 * parallelism is an OpenMP loop over independent (stream, chunk) units, which does not change
 * any output byte.
 */
#include "zn_oracle.h"

#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define ANS_SCALE 12
#define ANS_M (1u << ANS_SCALE)
#define ANS_L (1u << 15)
#define LANES 8
#define STEPS 16
#define ROUND (LANES * STEPS)

static int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }
static int64_t align8(int64_t x) { return (x + 7) & ~(int64_t)7; }

/* ---- reorder: src/cuzipnn/_kernels.py:17-31 ---------------------------------------------- */

uint64_t orc_reorder(uint64_t u, int w) {
    uint64_t exp = (u >> (w - 9)) & 0xFF;
    uint64_t sign = u >> (w - 1);
    uint64_t mant = u & ((1ull << (w - 9)) - 1);
    return (exp << (w - 8)) | (sign << (w - 9)) | mant;
}

uint64_t orc_revert(uint64_t u, int w) {
    uint64_t exp = u >> (w - 8);
    uint64_t sign = (u >> (w - 9)) & 1;
    uint64_t mant = u & ((1ull << (w - 9)) - 1);
    return (sign << (w - 1)) | (exp << (w - 9)) | mant;
}

static uint64_t load_elem(const uint8_t *p, int k) {
    uint64_t u = 0;
    for (int b = 0; b < k; b++) u |= (uint64_t)p[b] << (8 * b);
    return u;
}

/* ---- split / merge / copy: src/cuzipnn/_kernels.py:34-131 --------------------------------- */

void orc_split(const uint8_t *x, int64_t n, int k, int reorder, uint8_t *planar, int64_t stride) {
    for (int64_t e = 0; e < n; e++) {
        uint64_t u = load_elem(x + e * k, k);
        if (reorder) u = orc_reorder(u, 8 * k);
        for (int b = 0; b < k; b++) planar[b * stride + e] = (uint8_t)(u >> (8 * b));
    }
}

void orc_merge(const int64_t *src_tbl, const uint8_t *base, uint8_t *out, int64_t n, int k,
               int64_t chunk_bytes, int reorder) {
    int64_t nch = cdiv(n, chunk_bytes);
    for (int64_t e = 0; e < n; e++) {
        int64_t j = e / chunk_bytes, o = e - j * chunk_bytes;
        uint64_t u = 0;
        for (int b = 0; b < k; b++) u |= (uint64_t)base[src_tbl[b * nch + j] + o] << (8 * b);
        if (reorder) u = orc_revert(u, 8 * k);
        for (int b = 0; b < k; b++) out[e * k + b] = (uint8_t)(u >> (8 * b));
    }
}

void orc_copy_chunks(const uint8_t *src_base, const int64_t *src_off, uint8_t *dst_base,
                     const int64_t *dst_off, const int64_t *nbytes, int64_t count, int pad) {
    for (int64_t i = 0; i < count; i++) {
        int64_t nb = nbytes[i];
        if (nb <= 0) continue;
        memcpy(dst_base + dst_off[i], src_base + src_off[i], (size_t)nb);
        if (pad)
            for (int64_t q = nb; q < align8(nb); q++) dst_base[dst_off[i] + q] = 0;
    }
}

/* ---- CRC-32 (reflected 0x04C11DB7 = 0xEDB88320, init/xorout 0xFFFFFFFF) ------------------- */

static uint32_t crc_table[256];
static int crc_table_ready;

static void crc_init(void) {
    if (crc_table_ready) return;
    for (uint32_t i = 0; i < 256; i++) {
        uint32_t c = i;
        for (int b = 0; b < 8; b++) c = (c >> 1) ^ (0xEDB88320u & (0u - (c & 1u)));
        crc_table[i] = c;
    }
    crc_table_ready = 1;
}

uint32_t orc_crc32(uint32_t crc, const uint8_t *p, int64_t n) {
    crc_init();
    uint32_t c = ~crc;
    for (int64_t i = 0; i < n; i++) c = crc_table[(c ^ p[i]) & 0xFF] ^ (c >> 8);
    return ~c;
}

void orc_crc32_segments(const uint8_t *p, int64_t n, int64_t seg, uint32_t *out) {
    crc_init();
    int64_t m = cdiv(n, seg);
#pragma omp parallel for schedule(dynamic, 16)
    for (int64_t i = 0; i < m; i++) {
        int64_t len = (i == m - 1) ? n - i * seg : seg;
        out[i] = orc_crc32(0, p + i * seg, len);
    }
}

/* ---- sub-chunk count: src/cuzipnn/_codec.py:83-86 ---------------------------------------- */

int orc_sub_chunks(int64_t chunk_bytes, int64_t sub_chunk_bytes) {
    int64_t q = cdiv(chunk_bytes, sub_chunk_bytes) - 1; /* (q).bit_length() */
    int bl = 0;
    while (q > 0) { bl++; q >>= 1; }
    int64_t count = (int64_t)1 << bl;
    if (count < 4) count = 4;
    if (count > 64) count = 64;
    return (int)count;
}

/* ---- ZNR2 rANS payload ------------------------------------------------------------------- */

void orc_normalize(const uint32_t c[256], int64_t m, uint32_t f[256]) {
    int np = 0, smax = -1;
    uint32_t cmax = 0;
    for (int s = 0; s < 256; s++) {
        f[s] = 0;
        if (c[s]) {
            np++;
            if (c[s] > cmax) { cmax = c[s]; smax = s; }
        }
    }
    if (np == 0) return;
    if (np == 1) { f[smax] = ANS_M; return; }
    int64_t sum = 0;
    for (int s = 0; s < 256; s++) {
        if (!c[s]) continue;
        uint64_t q = ((uint64_t)c[s] * ANS_M + (uint64_t)(m / 2)) / (uint64_t)m;
        f[s] = q < 1 ? 1 : (uint32_t)q;
        sum += f[s];
    }
    int64_t d = (int64_t)ANS_M - sum;
    if ((int64_t)f[smax] + d >= 1) { f[smax] = (uint32_t)((int64_t)f[smax] + d); return; }
    sum = 0;
    for (int s = 0; s < 256; s++) {
        if (!c[s]) continue;
        f[s] = 1 + (uint32_t)(((uint64_t)c[s] * (uint64_t)(ANS_M - np)) / (uint64_t)m);
        sum += f[s];
    }
    f[smax] += (uint32_t)((int64_t)ANS_M - sum);
}

typedef struct {
    int64_t sc;  /* sub-chunk length in symbols (multiple of 128) */
    int nu;      /* non-empty sub-chunks */
    int lw;      /* bytes per stream-length field (one field per state) */
} ans_geom;

static ans_geom geom(int64_t m, int n_sub) {
    ans_geom g;
    g.sc = cdiv(cdiv(m, n_sub), ROUND) * ROUND;
    g.nu = (int)cdiv(m, g.sc);
    g.lw = g.sc / LANES < 65536 ? 2 : 4; /* a state emits at most one word per symbol */
    return g;
}

static int64_t table_bytes(int np) { return (2 + 32 + (12 * np + 7) / 8 + 3) & ~(int64_t)3; }

static int64_t lengths_bytes(ans_geom g) { return ((int64_t)g.nu * LANES * g.lw + 3) & ~(int64_t)3; }

static int64_t meta_bytes(int np, ans_geom g) {
    return table_bytes(np) + lengths_bytes(g) + (int64_t)g.nu * LANES * 4;
}

int64_t orc_ans_max_payload(int64_t m, int n_sub) {
    /* Any unit of at most m symbols: at most n_sub streams with 4-byte lengths, one word per
     * symbol.  (A shorter unit can have more sub-chunks than a full one.) */
    return table_bytes(256) + 4 * (int64_t)LANES * n_sub + (int64_t)LANES * 4 * n_sub + 2 * m;
}

static void put16(uint8_t *p, uint32_t v) { p[0] = (uint8_t)v; p[1] = (uint8_t)(v >> 8); }
static void put32(uint8_t *p, uint32_t v) {
    for (int i = 0; i < 4; i++) p[i] = (uint8_t)(v >> (8 * i));
}
static uint32_t get16(const uint8_t *p) { return p[0] | ((uint32_t)p[1] << 8); }
static uint32_t get32(const uint8_t *p) {
    return p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

int64_t orc_ans_encode(const uint8_t *sym, int64_t m, int n_sub, uint8_t *out, int64_t cap) {
    if (m < 1 || n_sub < 4 || n_sub > 64 || (n_sub & (n_sub - 1))) return -2;
    uint32_t cnt[256] = {0}, f[256], cum[257];
    for (int64_t i = 0; i < m; i++) cnt[sym[i]]++;
    orc_normalize(cnt, m, f);
    int np = 0;
    cum[0] = 0;
    for (int s = 0; s < 256; s++) { cum[s + 1] = cum[s] + f[s]; np += f[s] > 0; }

    ans_geom g = geom(m, n_sub);
    int64_t tb = table_bytes(np), mb = meta_bytes(np, g);
    if (cap < mb) return -1;
    memset(out, 0, (size_t)mb);
    int t = 0;
    while ((1 << t) < n_sub) t++;
    out[0] = (uint8_t)t;
    out[1] = 0;
    int k = 0;
    for (int s = 0; s < 256; s++) {
        if (!f[s]) continue;
        out[2 + (s >> 3)] |= (uint8_t)(1u << (s & 7));
        uint32_t v = f[s] - 1;
        for (int bit = 0; bit < 12; bit++)
            if (v >> bit & 1) {
                int64_t pos = 12 * (int64_t)k + bit;
                out[34 + (pos >> 3)] |= (uint8_t)(1u << (pos & 7));
            }
        k++;
    }
    uint8_t *lens = out + tb;
    uint8_t *states = lens + lengths_bytes(g);
    int64_t wpos = mb; /* byte offset where the next stream goes */

    /* One word list per state; words are produced last-first and stored first-last. */
    int64_t per = g.sc / LANES;
    uint16_t *tmp = (uint16_t *)malloc(sizeof(uint16_t) * (size_t)(LANES * per + 1));
    for (int gi = 0; gi < g.nu; gi++) {
        int64_t base = (int64_t)gi * g.sc;
        int64_t len = m - base < g.sc ? m - base : g.sc;
        int64_t rounds = cdiv(len, ROUND);
        uint32_t x[LANES];
        int64_t nw[LANES];
        for (int l = 0; l < LANES; l++) { x[l] = ANS_L; nw[l] = 0; }
        for (int64_t r = rounds - 1; r >= 0; r--) {
            for (int i = STEPS - 1; i >= 0; i--) {
                for (int l = 0; l < LANES; l++) {
                    int64_t p = r * ROUND + l * STEPS + i;
                    if (p >= len) continue;
                    int s = sym[base + p];
                    if ((x[l] >> 19) >= f[s]) { /* x >= f * 2^19 = ((L >> 12) << 16) * f */
                        tmp[l * per + nw[l]++] = (uint16_t)(x[l] & 0xFFFF);
                        x[l] >>= 16;
                    }
                    x[l] = (x[l] / f[s]) * ANS_M + x[l] % f[s] + cum[s];
                }
            }
        }
        for (int l = 0; l < LANES; l++) {
            if (wpos + 2 * nw[l] > cap) { free(tmp); return -1; }
            for (int64_t q = 0; q < nw[l]; q++) put16(out + wpos + 2 * q, tmp[l * per + nw[l] - 1 - q]);
            wpos += 2 * nw[l];
            int64_t fi = (int64_t)gi * LANES + l;
            if (g.lw == 2) put16(lens + 2 * fi, (uint32_t)nw[l]);
            else put32(lens + 4 * fi, (uint32_t)nw[l]);
            put32(states + 4 * fi, x[l]);
        }
    }
    free(tmp);
    return wpos;
}

int orc_ans_decode(const uint8_t *pl, int64_t size, int64_t m, uint8_t *out) {
    if (m < 1 || size < 34) return -1;
    int t = pl[0];
    if (t < 2 || t > 6 || pl[1] != 0) return -2;
    uint32_t f[256], cum[257];
    int np = 0;
    for (int s = 0; s < 256; s++) np += (pl[2 + (s >> 3)] >> (s & 7)) & 1;
    if (np == 0) return -3;
    int64_t tb = table_bytes(np);
    ans_geom g = geom(m, 1 << t);
    int64_t mb = meta_bytes(np, g);
    if (size < mb) return -4;
    int k = 0;
    cum[0] = 0;
    for (int s = 0; s < 256; s++) {
        f[s] = 0;
        if ((pl[2 + (s >> 3)] >> (s & 7)) & 1) {
            uint32_t v = 0;
            for (int bit = 0; bit < 12; bit++) {
                int64_t pos = 12 * (int64_t)k + bit;
                v |= (uint32_t)((pl[34 + (pos >> 3)] >> (pos & 7)) & 1) << bit;
            }
            f[s] = v + 1;
            k++;
        }
        cum[s + 1] = cum[s] + f[s];
    }
    if (cum[256] != ANS_M) return -5;
    uint8_t slot_sym[ANS_M];
    for (int s = 0; s < 256; s++)
        for (uint32_t q = cum[s]; q < cum[s + 1]; q++) slot_sym[q] = (uint8_t)s;
    const uint8_t *lens = pl + tb;
    const uint8_t *states = lens + lengths_bytes(g);
    int64_t spos = mb;
    for (int gi = 0; gi < g.nu; gi++) {
        const uint8_t *ws[LANES];
        int64_t nw[LANES], ptr[LANES];
        uint32_t x[LANES];
        for (int l = 0; l < LANES; l++) {
            int64_t fi = (int64_t)gi * LANES + l;
            nw[l] = g.lw == 2 ? get16(lens + 2 * fi) : get32(lens + 4 * fi);
            if (spos + 2 * nw[l] > size) return -6;
            ws[l] = pl + spos;
            spos += 2 * nw[l];
            ptr[l] = 0;
            x[l] = get32(states + 4 * fi);
            if (x[l] < ANS_L || x[l] >= 0x80000000u) return -7;
        }
        int64_t base = (int64_t)gi * g.sc;
        int64_t len = m - base < g.sc ? m - base : g.sc;
        int64_t rounds = cdiv(len, ROUND);
        for (int64_t r = 0; r < rounds; r++) {
            for (int i = 0; i < STEPS; i++) {
                for (int l = 0; l < LANES; l++) {
                    int64_t p = r * ROUND + l * STEPS + i;
                    if (p >= len) continue;
                    uint32_t slot = x[l] & (ANS_M - 1);
                    int s = slot_sym[slot];
                    out[base + p] = (uint8_t)s;
                    x[l] = f[s] * (x[l] >> ANS_SCALE) + slot - cum[s];
                    if (x[l] < ANS_L) {
                        if (ptr[l] >= nw[l]) return -8;
                        x[l] = (x[l] << 16) | get16(ws[l] + 2 * ptr[l]);
                        ptr[l]++;
                    }
                }
            }
        }
        for (int l = 0; l < LANES; l++)
            if (ptr[l] != nw[l] || x[l] != ANS_L) return -9;
    }
    return spos == size ? 0 : -10;
}

/* ---- container: src/cuzipnn/_codec.py:1-21, :89-93, :270-306, :361-403, :416-542 ---------- */

int64_t orc_blob_bound(int64_t n, int k, int ndim, int64_t chunk_bytes) {
    int64_t nch = cdiv(n, chunk_bytes), total = (int64_t)k * nch;
    int64_t head = align8(24 + 8 * (int64_t)ndim + 8 * total);
    int64_t data = 0;
    if (nch) data = (int64_t)k * ((nch - 1) * align8(chunk_bytes) + align8(n - (nch - 1) * chunk_bytes));
    int64_t stored = 24 + 8 * (int64_t)ndim + n * k;
    return head + data > stored ? head + data : stored;
}

static void write_header(uint8_t *out, int version, int code, int ndim, int flags,
                         uint32_t chunk_bytes, uint32_t n_comp, uint64_t n, const int64_t *shape) {
    memcpy(out, "ZNNG", 4);
    out[4] = (uint8_t)version;
    out[5] = (uint8_t)code;
    out[6] = (uint8_t)ndim;
    out[7] = (uint8_t)flags;
    put32(out + 8, chunk_bytes);
    put32(out + 12, n_comp);
    for (int i = 0; i < 8; i++) out[16 + i] = (uint8_t)(n >> (8 * i));
    for (int d = 0; d < ndim; d++)
        for (int i = 0; i < 8; i++) out[24 + 8 * d + i] = (uint8_t)((uint64_t)shape[d] >> (8 * i));
}

int64_t orc_compress(const uint8_t *x, int64_t n, int k, int dtype_code, int reorder, int ndim,
                     const int64_t *shape, int64_t chunk_bytes, int n_sub, double threshold,
                     int64_t min_compress_bytes, int version, uint8_t *out, int64_t cap,
                     int threads) {
    int64_t header = 24 + 8 * (int64_t)ndim;
    if (n * k < min_compress_bytes || n == 0) {
        int stored = n * k < min_compress_bytes;
        if (cap < header + n * k) return -1;
        write_header(out, version, dtype_code, ndim, stored ? 2 : (reorder ? 1 : 0),
                     stored ? 0u : (uint32_t)chunk_bytes, 0, (uint64_t)n, shape);
        memcpy(out + header, x, (size_t)(n * k));
        return header + n * k;
    }
    int64_t nch = cdiv(n, chunk_bytes), total = (int64_t)k * nch;
    int64_t stride = nch * chunk_bytes;
    uint8_t *planar = (uint8_t *)malloc((size_t)(total * chunk_bytes));
    orc_split(x, n, k, reorder, planar, stride);

    int64_t last = n - (nch - 1) * chunk_bytes;
    int64_t slot = align8(orc_ans_max_payload(chunk_bytes, n_sub));
    uint8_t *comp = (uint8_t *)malloc((size_t)(total * slot));
    int64_t *comp_bytes = (int64_t *)malloc(sizeof(int64_t) * (size_t)total);
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t i = 0; i < total; i++) {
        int64_t b = i / nch, j = i % nch;
        int64_t raw = j == nch - 1 ? last : chunk_bytes;
        comp_bytes[i] = orc_ans_encode(planar + b * stride + j * chunk_bytes, raw, n_sub,
                                       comp + i * slot, slot);
    }
    /* _codec.py:361-372: keep a chunk compressed only if it is below trunc(raw * threshold). */
    int64_t *stored = (int64_t *)malloc(sizeof(int64_t) * (size_t)total);
    int64_t n_comp = 0, data = 0;
    for (int64_t i = 0; i < total; i++) {
        int64_t j = i % nch;
        int64_t raw = j == nch - 1 ? last : chunk_bytes;
        int64_t thr = (int64_t)((double)raw * threshold);
        int64_t c = comp_bytes[i] >= 0 ? comp_bytes[i] : ((int64_t)1 << 24);
        int use = c < thr;
        stored[i] = use ? c : raw;
        comp_bytes[i] = use;
        n_comp += use;
        data += align8(stored[i]);
    }
    int64_t sizes_off = header, idx_off = sizes_off + 4 * total;
    int64_t data_off = align8(idx_off + 4 * n_comp);
    int64_t size = data_off + data;
    if (size > cap) { free(planar); free(comp); free(comp_bytes); free(stored); return -1; }
    memset(out, 0, (size_t)data_off);
    write_header(out, version, dtype_code, ndim, reorder ? 1 : 0, (uint32_t)chunk_bytes,
                 (uint32_t)n_comp, (uint64_t)n, shape);
    int64_t q = 0, pos = data_off;
    for (int64_t i = 0; i < total; i++) {
        put32(out + sizes_off + 4 * i, (uint32_t)stored[i]);
        if (comp_bytes[i]) put32(out + idx_off + 4 * q++, (uint32_t)i);
        int64_t b = i / nch, j = i % nch;
        const uint8_t *src = comp_bytes[i] ? comp + i * slot : planar + b * stride + j * chunk_bytes;
        memcpy(out + pos, src, (size_t)stored[i]);
        memset(out + pos + stored[i], 0, (size_t)(align8(stored[i]) - stored[i]));
        pos += align8(stored[i]);
    }
    free(planar);
    free(comp);
    free(comp_bytes);
    free(stored);
    return size;
}

int orc_decompress(const uint8_t *blob, int64_t size, uint8_t *out, int64_t out_bytes,
                   int version, int threads) {
    if (size < 24 || memcmp(blob, "ZNNG", 4) != 0 || blob[4] != version) return -1;
    int code = blob[5], ndim = blob[6], flags = blob[7];
    if (code < 1 || code > 16) return -1;
    static const int ksize[17] = {0, 1, 1, 1, 2, 4, 8, 2, 2, 4, 8, 1, 1, 2, 4, 8, 8};
    int k = ksize[code];
    int64_t chunk_bytes = get32(blob + 8), n_comp = get32(blob + 12);
    int64_t n = 0;
    for (int i = 0; i < 8; i++) n |= (int64_t)blob[16 + i] << (8 * i);
    int64_t header = 24 + 8 * (int64_t)ndim;
    if (size < header || out_bytes != n * k) return -2;
    if (flags & 2) {
        if (size < header + n * k) return -3;
        memcpy(out, blob + header, (size_t)(n * k));
        return 0;
    }
    if (n == 0) return 0;
    if (chunk_bytes <= 0) return -4;
    int reorder = flags & 1;
    int64_t nch = cdiv(n, chunk_bytes), total = (int64_t)k * nch;
    int64_t sizes_off = header, idx_off = sizes_off + 4 * total;
    int64_t data_off = align8(idx_off + 4 * n_comp);
    if (size < data_off) return -5;
    int64_t *src = (int64_t *)malloc(sizeof(int64_t) * (size_t)total);
    uint8_t *is_comp = (uint8_t *)calloc((size_t)total, 1);
    int64_t pos = data_off;
    for (int64_t i = 0; i < total; i++) {
        src[i] = pos;
        pos += align8((int64_t)(int32_t)get32(blob + sizes_off + 4 * i));
    }
    for (int64_t q = 0; q < n_comp; q++) {
        int64_t i = (int32_t)get32(blob + idx_off + 4 * q);
        if (i < 0 || i >= total) { free(src); free(is_comp); return -6; }
        is_comp[i] = 1;
    }
    int64_t stride = nch * chunk_bytes, last = n - (nch - 1) * chunk_bytes;
    uint8_t *planar = (uint8_t *)malloc((size_t)(total * chunk_bytes));
    int err = 0;
#ifdef _OPENMP
    if (threads > 0) omp_set_num_threads(threads);
#endif
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t i = 0; i < total; i++) {
        int64_t b = i / nch, j = i % nch;
        int64_t raw = j == nch - 1 ? last : chunk_bytes;
        int64_t st = (int32_t)get32(blob + sizes_off + 4 * i);
        uint8_t *dst = planar + b * stride + j * chunk_bytes;
        if (src[i] + st > size) { err = -7; continue; }
        if (is_comp[i]) {
            if (orc_ans_decode(blob + src[i], st, raw, dst) != 0) err = -8;
        } else {
            if (st != raw) { err = -9; continue; }
            memcpy(dst, blob + src[i], (size_t)raw);
        }
    }
    if (!err) {
        int64_t *tbl = (int64_t *)malloc(sizeof(int64_t) * (size_t)total);
        for (int64_t i = 0; i < total; i++) tbl[i] = (i / nch) * stride + (i % nch) * chunk_bytes;
        orc_merge(tbl, planar, out, n, k, chunk_bytes, reorder);
        free(tbl);
    }
    free(planar);
    free(src);
    free(is_comp);
    return err;
}
