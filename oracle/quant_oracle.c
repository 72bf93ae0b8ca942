/*
 * CPU oracle: C restatement of the reference bridge's host quantisers -- TEST INFRASTRUCTURE ONLY.
 *
 * Only tests/ and bench.py's CPU-baseline leg load this (oracle/_build/libquant_oracle.so).
 * Compiled with -ffp-contract=off so that every source-level fp32 operation rounds once, which
 * is the IEEE reading of the reference source text:
 *   metal_kan_quantize_int8     metal_kans/kernels/metal_kan_bridge.mm:4177-4211
 *   metal_kan_dequantize_int8   metal_kan_bridge.mm:4213-4232
 *   metal_kan_quantize_int4     metal_kan_bridge.mm:4234-4275
 *   metal_kan_dequantize_int4   metal_kan_bridge.mm:4278-4302
 *   metal_kan_quantize_ternary  metal_kan_bridge.mm:4634-4682
 *   metal_kan_quantize_int2     metal_kan_bridge.mm:4735-4788
 *   dequantize_ternary_fast / dequantize_int2_fast   metal_kans/kernels/fused_kan.metal:2392-2441
 * The function names carry an "oracle_" prefix so they can never be mistaken for the product's
 * exports of the same reference names.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static void minmax(const float* g, int n, float* mn, float* mx) {
    float a = g[0], b = g[0];
    for (int i = 1; i < n; ++i) {
        if (g[i] < a) a = g[i];
        if (g[i] > b) b = g[i];
    }
    *mn = a;
    *mx = b;
}

static int qclamp(float v, int maxq) {
    int q = (int)v;
    if (q < 0) q = 0;
    else if (q > maxq) q = maxq;
    return q;
}

int oracle_quantize_affine(const float* w, uint8_t* q, float* s, float* b, int groups, int gs,
                           int bits) {
    if (!w || !q || !s || !b || groups <= 0 || gs <= 0) return -1;
    const int maxq = (1 << bits) - 1;
    for (int g = 0; g < groups; ++g) {
        const float* grp = w + (size_t)g * gs;
        float mn, mx;
        minmax(grp, gs, &mn, &mx);
        float range = mx - mn;
        if (range < 1e-7f) range = 1e-7f;
        float scale = range / (float)maxq;
        s[g] = scale;
        b[g] = mn;
        float inv = 1.0f / scale;
        if (bits == 8) {
            for (int i = 0; i < gs; ++i) {
                float d = grp[i] - mn;
                float p = d * inv;
                q[(size_t)g * gs + i] = (uint8_t)qclamp(p + 0.5f, maxq);
            }
        } else {
            for (int i = 0; i < gs / 2; ++i) {
                float d0 = grp[2 * i] - mn, d1 = grp[2 * i + 1] - mn;
                float p0 = d0 * inv, p1 = d1 * inv;
                int q0 = qclamp(p0 + 0.5f, maxq), q1 = qclamp(p1 + 0.5f, maxq);
                q[(size_t)g * (gs / 2) + i] = (uint8_t)(q0 | (q1 << 4));
            }
        }
    }
    return 0;
}

int oracle_dequantize_affine(const uint8_t* q, const float* s, const float* b, float* out,
                             int groups, int gs, int bits) {
    if (!q || !s || !b || !out || groups <= 0 || gs <= 0) return -1;
    for (int g = 0; g < groups; ++g) {
        for (int i = 0; i < gs; ++i) {
            int v;
            if (bits == 8) v = q[(size_t)g * gs + i];
            else {
                uint8_t byte = q[(size_t)g * (gs / 2) + i / 2];
                v = (i & 1) ? (byte >> 4) & 0xF : byte & 0xF;
            }
            float m = (float)v * s[g];
            out[(size_t)g * gs + i] = m + b[g];
        }
    }
    return 0;
}

int oracle_quantize_ternary(const float* W, uint32_t* P, float* s, int D_out, int K_dim, int gs) {
    if (!W || !P || !s || D_out <= 0 || K_dim <= 0 || gs <= 0) return -1;
    int words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
    memset(P, 0, (size_t)D_out * words * sizeof(uint32_t));
    for (int j = 0; j < D_out; ++j) {
        const float* row = W + (size_t)j * K_dim;
        for (int g = 0; g < G; ++g) {
            int st = g * gs, en = st + gs < K_dim ? st + gs : K_dim, cnt = en - st;
            double sum = 0.0;
            for (int k = st; k < en; ++k) sum += fabs((double)row[k]);
            float sc = (cnt > 0 && sum > 0.0) ? (float)(sum / cnt) : 1e-4f;
            s[(size_t)j * G + g] = sc;
            float inv = 1.0f / sc;
            for (int k = st; k < en; ++k) {
                float v = row[k] * inv;
                uint32_t c = 1;
                if (v < -0.5f) c = 0;
                else if (v > 0.5f) c = 2;
                P[(size_t)j * words + k / 16] |= c << ((k % 16) * 2);
            }
        }
    }
    return 0;
}

int oracle_quantize_int2(const float* W, uint32_t* P, float* s, const float* cb, int D_out,
                         int K_dim, int gs) {
    if (!W || !P || !s || !cb || D_out <= 0 || K_dim <= 0 || gs <= 0) return -1;
    int words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
    memset(P, 0, (size_t)D_out * words * sizeof(uint32_t));
    for (int j = 0; j < D_out; ++j) {
        const float* row = W + (size_t)j * K_dim;
        for (int g = 0; g < G; ++g) {
            int st = g * gs, en = st + gs < K_dim ? st + gs : K_dim;
            float mx = 0.0f;
            for (int k = st; k < en; ++k) {
                float a = fabsf(row[k]);
                if (a > mx) mx = a;
            }
            float sc = mx > 0.0f ? mx : 1e-4f;
            s[(size_t)j * G + g] = sc;
            float inv = 1.0f / sc;
            for (int k = st; k < en; ++k) {
                float v = row[k] * inv;
                int best = 0;
                float bd = fabsf(v - cb[0]);
                for (int c = 1; c < 4; ++c) {
                    float d = fabsf(v - cb[c]);
                    if (d < bd) {
                        bd = d;
                        best = c;
                    }
                }
                P[(size_t)j * words + k / 16] |= (uint32_t)best << ((k % 16) * 2);
            }
        }
    }
    return 0;
}

int oracle_dequantize_2bit(const uint32_t* P, const float* s, const float* cb, float* out,
                           int D_out, int K_dim, int gs) {
    /* cb == NULL: ternary decode (code-1, code 3 -> 0); else codebook decode. */
    if (!P || !s || !out || D_out <= 0 || K_dim <= 0 || gs <= 0) return -1;
    int words = (K_dim + 15) / 16, G = (K_dim + gs - 1) / gs;
    for (int j = 0; j < D_out; ++j)
        for (int k = 0; k < K_dim; ++k) {
            uint32_t c = (P[(size_t)j * words + k / 16] >> ((k % 16) * 2)) & 3u;
            float sc = s[(size_t)j * G + k / gs];
            float wv;
            if (cb) wv = cb[c];
            else wv = (c == 3) ? 0.0f : (float)c - 1.0f;
            out[(size_t)j * K_dim + k] = wv * sc;
        }
    return 0;
}
