/*
 * CPU restatement of the Espalier decode hot path.  TEST INFRASTRUCTURE ONLY: this file is the oracle the CUDA
 * kernels are checked against (tests/, the smoke check) and the timed CPU baseline of bench.py.  Nothing on the
 * product path links or calls it.
 *
 * Every function restates the arithmetic of the reference plugin (geodesa-ai/vllm-espalier) in plain C, in the same
 * order of floating-point operations where the reference fixes one, so that integer / byte / index results are
 * bit-exact and floating-point results are either bit-exact (rotations, codebooks, routing ids) or differ only by the
 * accumulation order of a dot product (layer outputs).
 *
 *   codebooks ............ vllm_espalier/csrc/experts_grouped.cuh:23-80   (cb_pair<1,3,6,7,22,23>)
 *   trellis geometry ..... vllm_espalier/csrc/experts_grouped.cuh:83-154  (Fmt::end, LaneMap, decode_tile)
 *   value -> (row, col) .. vllm_espalier/csrc/experts_grouped.cuh:330-339 (dequant_kernel store)
 *   FWHT-128 ............. vllm_espalier/csrc/dense.cu:43-54, experts.cu:79-90
 *   input rotation ....... vllm_espalier/csrc/dense.cu:92-108, experts.cu:97-115
 *   dense epilogue ....... vllm_espalier/csrc/dense.cu:120-128, 73-89
 *   gate/up epilogue ..... vllm_espalier/csrc/experts.cu:120-162 (act_mode 1, fp32 SwiGLU)
 *   down + combine ....... vllm_espalier/csrc/experts.cu:340-393
 *   grouping ............. vllm_espalier/csrc/experts.cu:23-76, route.cu:132-179
 *   routing .............. vllm_espalier/csrc/route.cu:49-128, with the logit reduction order of this project's
 *                          routing kernel (fp64 sums of fp32 products, fixed lane order; see orc_router_logit)
 *                          so ids are exact.
 *
 * Build: oracle/Makefile (gcc -O2 -fopenmp -shared).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define HAD_SCALE 0.08838834764831845f /* 1 / sqrt(128) as the reference's float literal */

/* ------------------------------------------------------------------------------------------------------------ */
/* IEEE helpers: exact fp16 / bf16 <-> float, round-to-nearest-even narrowing                                     */
/* ------------------------------------------------------------------------------------------------------------ */

float orc_h2f(uint16_t h) {
    const uint32_t s = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu, f;
    if (e == 0) {
        if (m == 0) {
            f = s;
        } else { /* subnormal: normalise */
            int sh = 0;
            while (!(m & 0x400u)) { m <<= 1; ++sh; }
            m &= 0x3ffu;
            f = s | ((uint32_t)(113 - sh) << 23) | (m << 13);
        }
    } else if (e == 31) {
        f = s | 0x7f800000u | (m << 13);
    } else {
        f = s | ((e + 112u) << 23) | (m << 13);
    }
    float r;
    memcpy(&r, &f, 4);
    return r;
}

/* Round a finite double to a binary format with p significant bits and minimum normal exponent emin (round to
 * nearest, ties to even), returning the rounded value as a double (exact). */
static double round_fmt(double v, int p, int emin) {
    if (v == 0.0 || !isfinite(v)) return v;
    int ex;
    frexp(v, &ex);                      /* v = m * 2^ex, 0.5 <= |m| < 1  => unit in last place 2^(ex - p) */
    int q = ex - p;
    if (q < emin - p + 1) q = emin - p + 1; /* subnormal range keeps the fixed quantum */
    double t = ldexp(v, -q);            /* exact */
    double r = nearbyint(t);            /* default rounding mode: to nearest, ties to even */
    return ldexp(r, q);
}

uint16_t orc_d2h(double v) {
    const uint16_t sign = signbit(v) ? 0x8000u : 0;
    if (isnan(v)) return 0x7e00u;
    double r = fabs(round_fmt(v, 11, -14));
    if (r >= 65536.0 || isinf(r)) return sign | 0x7c00u;
    if (r == 0.0) return sign;
    int ex;
    frexp(r, &ex);                      /* r = m 2^ex, value exponent E = ex - 1 */
    int E = ex - 1;
    if (E < -14) { /* subnormal: r = m * 2^-24 */
        return sign | (uint16_t)ldexp(r, 24);
    }
    uint32_t mant = (uint32_t)(ldexp(r, 10 - E) - 1024.0);
    return sign | (uint16_t)(((uint32_t)(E + 15) << 10) | mant);
}

uint16_t orc_f2h(float f) { return orc_d2h((double)f); }

float orc_bf2f(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float r;
    memcpy(&r, &u, 4);
    return r;
}

uint16_t orc_d2bf(double v) {
    if (isnan(v)) return 0x7fc0u;
    /* bf16: 8 significant bits, exponent range of fp32 */
    double r = round_fmt(v, 8, -126);
    float f = (float)r;                 /* exact: r has 8 significant bits */
    uint32_t u;
    memcpy(&u, &f, 4);
    if (fabs(r) >= 3.3961775292304e38) u = (u & 0x80000000u) | 0x7f800000u;
    return (uint16_t)(u >> 16);
}

uint16_t orc_f2bf(float f) { return orc_d2bf((double)f); }

/* ------------------------------------------------------------------------------------------------------------ */
/* Codebooks (experts_grouped.cuh:23-80): a 16-bit trellis state -> fp16 bits                                     */
/* ------------------------------------------------------------------------------------------------------------ */

/* fp16 (a + b) rounded to nearest even: the sum of two fp16 is exact in double. */
static uint16_t hadd(uint16_t a, uint16_t b) { return orc_d2h((double)orc_h2f(a) + (double)orc_h2f(b)); }

/* mcg, codebook 1: x = s * 0xCBAC1FED; x = (x & 0x8FFF8FFF) ^ 0x3B603B60; v = fp16(lo) + fp16(hi) */
uint16_t orc_mcg(uint32_t s) {
    uint32_t x = (s & 0xffffu) * 0xCBAC1FEDu;
    x = (x & 0x8FFF8FFFu) ^ 0x3B603B60u;
    return hadd((uint16_t)(x & 0xffffu), (uint16_t)(x >> 16));
}

/* int5 / int6 grid (codebooks 6 / 7, and their index forms 22 / 23): q = rintf(v * k) in fp32 with the reference's
 * constants k; the value is fp16(q * c), c = 3.94921875f / 15 or / 31 computed in fp32; the index form is fp16(q). */
static const float INT_K5 = 0x1.e62c10p+1f;
static const float INT_K6 = 0x1.f660bap+2f;

float orc_int_step(int cb) {
    volatile float top = (cb == 6 || cb == 22) ? 15.0f : 31.0f;   /* fp32 division, as the reference's constexpr */
    return 3.94921875f / top;
}

static float int_q(uint16_t v, int six) {
    const float k = six ? INT_K6 : INT_K5;
    volatile float p = orc_h2f(v) * k;  /* one fp32 rounding of the product */
    return rintf(p);                    /* ties to even */
}

/* E2M1 grid (codebook 3): |v| against C * {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5}, summing C * {.5,.5,.5,.5,1,1,2},
 * then v's sign bit OR'd in; C = 0.75. Every threshold, step and partial sum is exact in fp16, so the hfma2 chain is
 * the exact sum. */
static uint16_t e2m1(uint16_t m) {
    const double C = 0.75;
    const double a = fabs((double)orc_h2f(m));
    static const double th[7] = {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0};
    static const double st[7] = {0.5, 0.5, 0.5, 0.5, 1.0, 1.0, 2.0};
    double acc = 0.0;
    for (int i = 0; i < 7; ++i)
        if (a > th[i] * C) acc += st[i] * C;
    return orc_d2h(acc) | (m & 0x8000u);
}

uint16_t orc_codebook(int cb, uint32_t state) {
    const uint16_t m = orc_mcg(state);
    switch (cb) {
        case 1: return m;
        case 3: return e2m1(m);
        case 6: return orc_f2h(int_q(m, 0) * orc_int_step(6));
        case 7: return orc_f2h(int_q(m, 1) * orc_int_step(7));
        case 22: return orc_f2h(int_q(m, 0));
        case 23: return orc_f2h(int_q(m, 1));
        default: return 0xffffu;
    }
}

void orc_codebook_table(int cb, uint16_t* out) {
#pragma omp parallel for schedule(static)
    for (int s = 0; s < 65536; ++s) out[s] = orc_codebook(cb, (uint32_t)s);
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Trellis geometry (Appendix of the format; experts_grouped.cuh:83-154, 330-339)                                 */
/* A tile of 16x16 weights is a circular MSB-first bitstream of 256*K bits held in 8*K uint32 words (int16 pairs,   */
/* little-endian). Value p's state is the 16 bits ending just before stream position (p + 1) * K.                 */
/* ------------------------------------------------------------------------------------------------------------ */

static inline uint32_t stream_bit(const uint32_t* w, int b) { return (w[b >> 5] >> (31 - (b & 31))) & 1u; }

uint32_t orc_state(const uint32_t* tile, int K, int p) {
    const int nbits = 256 * K;
    const int end = (p + 1) * K;
    uint32_t s = 0;
    for (int i = 0; i < 16; ++i) {
        int b = end - 16 + i;
        b = ((b % nbits) + nbits) % nbits;
        s = (s << 1) | stream_bit(tile, b);
    }
    return s;
}

/* position of value p inside its tile: p = 8 * lane + j, lane = 4g + t */
void orc_value_pos(int p, int* row, int* col) {
    const int lane = p >> 3, j = p & 7, g = lane >> 2, t = lane & 3;
    *row = 2 * t + 8 * ((j >> 1) & 1) + (j & 1);
    *col = g + 8 * (j >> 2);
}

/* trellis int16 [Kin/16][N/16][16*K] -> state of every weight, uint16 [Kin][N] */
void orc_states(const int16_t* T, int Kin, int N, int K, uint16_t* S) {
    const int KT = Kin / 16, NT = N / 16, TW = 8 * K;
#pragma omp parallel for schedule(static)
    for (int kt = 0; kt < KT; ++kt)
        for (int nt = 0; nt < NT; ++nt) {
            const uint32_t* w = (const uint32_t*)(T + ((size_t)kt * NT + nt) * 2 * TW);
            for (int p = 0; p < 256; ++p) {
                int r, c;
                orc_value_pos(p, &r, &c);
                S[(size_t)(kt * 16 + r) * N + nt * 16 + c] = (uint16_t)orc_state(w, K, p);
            }
        }
}

/* W fp16 bits [Kin][N] = codebook(state) (dequant_kernel, experts_grouped.cuh:321-340) */
int orc_dequant(const int16_t* T, int Kin, int N, int K, int cb, uint16_t* W) {
    if (Kin % 16 || N % 16 || K < 1 || K > 8) return -1;
    uint16_t* tab = (uint16_t*)malloc(65536 * sizeof(uint16_t));
    if (!tab) return -2;
    orc_codebook_table(cb, tab);
    if (tab[0] == 0xffffu && cb != 1) { free(tab); return -3; }
    const int KT = Kin / 16, NT = N / 16, TW = 8 * K;
#pragma omp parallel for schedule(static)
    for (int kt = 0; kt < KT; ++kt)
        for (int nt = 0; nt < NT; ++nt) {
            const uint32_t* w = (const uint32_t*)(T + ((size_t)kt * NT + nt) * 2 * TW);
            for (int p = 0; p < 256; ++p) {
                int r, c;
                orc_value_pos(p, &r, &c);
                W[(size_t)(kt * 16 + r) * N + nt * 16 + c] = tab[orc_state(w, K, p)];
            }
        }
    free(tab);
    return 0;
}

/* ------------------------------------------------------------------------------------------------------------ */
/* orc_dequant widened to fp32, for the timed CPU baseline (the reference's decode-then-matmul path restated on the */
/* host): the same states, each cut from a 64-bit window of two stream words instead of bit by bit, and the        */
/* codebook as an fp32 table, so the host decode is not a bit-serial strawman. tests/test_oracle.py checks it      */
/* against orc_dequant for every compiled (codebook, width) pair, bit for bit.                                     */
/* ------------------------------------------------------------------------------------------------------------ */
int orc_dequant_f32(const int16_t* T, int Kin, int N, int K, int cb, float* W) {
    if (Kin % 16 || N % 16 || K < 1 || K > 8) return -1;
    uint16_t* tab = (uint16_t*)malloc(65536 * sizeof(uint16_t));
    float* ftab = (float*)malloc(65536 * sizeof(float));
    if (!tab || !ftab) { free(tab); free(ftab); return -2; }
    orc_codebook_table(cb, tab);
    if (tab[0] == 0xffffu && cb != 1) { free(tab); free(ftab); return -3; }
    for (int i = 0; i < 65536; ++i) ftab[i] = orc_h2f(tab[i]);
    int off[256];
    for (int p = 0; p < 256; ++p) {
        int r, c;
        orc_value_pos(p, &r, &c);
        off[p] = r * N + c;
    }
    const int KT = Kin / 16, NT = N / 16, TW = 8 * K, nbits = 256 * K;
#pragma omp parallel for schedule(static)
    for (int kt = 0; kt < KT; ++kt)
        for (int nt = 0; nt < NT; ++nt) {
            const uint32_t* w = (const uint32_t*)(T + ((size_t)kt * NT + nt) * 2 * TW);
            float* out = W + (size_t)kt * 16 * N + nt * 16;
            for (int p = 0; p < 256; ++p) {
                int b = (p + 1) * K - 16;                       /* the state's first stream bit (circular) */
                if (b < 0) b += nbits;
                const int wi = b >> 5, sh = b & 31;
                const uint64_t x = ((uint64_t)w[wi] << 32) | w[(wi + 1) % TW];   /* 64 stream bits, MSB first */
                out[off[p]] = ftab[(x >> (48 - sh)) & 0xffffu];
            }
        }
    free(tab);
    free(ftab);
    return 0;
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Hadamard-128 with the reference's butterfly order (dense.cu:43-54): lane L holds v[4L..4L+3]; H4 in registers,  */
/* then xor-partner stages 1, 2, 4, 8, 16 across lanes (lower lane a + b, upper lane a - b).                       */
/* ------------------------------------------------------------------------------------------------------------ */

void orc_fwht128(float* v) {
    for (int L = 0; L < 32; ++L) {
        float* q = v + 4 * L;
        const float a = q[0] + q[1], b = q[0] - q[1], c = q[2] + q[3], d = q[2] - q[3];
        q[0] = a + c; q[1] = b + d; q[2] = a - c; q[3] = b - d;
    }
    for (int m = 1; m < 32; m <<= 1)
        for (int L = 0; L < 32; ++L) {
            if (L & m) continue;
            for (int j = 0; j < 4; ++j) {
                const float a = v[4 * L + j], b = v[4 * (L | m) + j];
                v[4 * L + j] = a + b;
                v[4 * (L | m) + j] = a - b;
            }
        }
}

/* xh fp16 [M][K] = fp16(FWHT(x * suh) * HAD) per 128-block (dense.cu:92-108); x given as exact float values. */
void orc_rotate(const float* x, int M, int K, const uint16_t* suh, uint16_t* xh) {
    for (int r = 0; r < M; ++r)
        for (int b = 0; b < K; b += 128) {
            float v[128];
            for (int i = 0; i < 128; ++i) {
                const float p = x[(size_t)r * K + b + i] * orc_h2f(suh[b + i]);   /* __fmul_rn */
                v[i] = p;
            }
            orc_fwht128(v);
            for (int i = 0; i < 128; ++i) {
                volatile float t = v[i] * HAD_SCALE;
                xh[(size_t)r * K + b + i] = orc_f2h(t);
            }
        }
}

/* The dense layer's finished fp32 outputs (dense.cu:120-128) from xh (fp16 bits) and W (fp16 bits):
 * acc[m][n] = sum_k xh * W accumulated in double (the GPU sums in fp32 on tensor cores: compare within tolerance),
 * then per 128-block FWHT, * scale, * (HAD * svh). y fp32 [M][N]. */
void orc_dense(const uint16_t* xh, const uint16_t* W, int M, int K, int N, const uint16_t* svh, float scale,
               float* y) {
    float* wf = (float*)malloc((size_t)K * N * sizeof(float));
    for (size_t i = 0; i < (size_t)K * N; ++i) wf[i] = orc_h2f(W[i]);
#pragma omp parallel for schedule(static)
    for (int m = 0; m < M; ++m) {
        double* acc = (double*)calloc((size_t)N, sizeof(double));
        for (int k = 0; k < K; ++k) {
            const double a = orc_h2f(xh[(size_t)m * K + k]);
            if (a == 0.0) continue;
            const float* wr = wf + (size_t)k * N;
            for (int n = 0; n < N; ++n) acc[n] += a * (double)wr[n];
        }
        for (int b = 0; b < N; b += 128) {
            float v[128];
            for (int i = 0; i < 128; ++i) v[i] = (float)acc[b + i];
            orc_fwht128(v);
            for (int i = 0; i < 128; ++i) {
                volatile float s1 = v[i] * scale;
                volatile float hs = HAD_SCALE * orc_h2f(svh[b + i]);
                volatile float o = s1 * hs;
                y[(size_t)m * N + b + i] = o;
            }
        }
        free(acc);
    }
    free(wf);
}

/* y fp16 = fp16(FWHT(x * pre) * HAD * post) (dense.cu:242-265); pre / post may be NULL. x fp16 bits [M][K]. */
void orc_had(const uint16_t* x, int M, int K, const uint16_t* pre, const uint16_t* post, uint16_t* y) {
    for (int r = 0; r < M; ++r)
        for (int b = 0; b < K; b += 128) {
            float v[128];
            for (int i = 0; i < 128; ++i) {
                float a = orc_h2f(x[(size_t)r * K + b + i]);
                if (pre) { volatile float p = a * orc_h2f(pre[b + i]); a = p; }
                v[i] = a;
            }
            orc_fwht128(v);
            for (int i = 0; i < 128; ++i) {
                volatile float t = v[i] * HAD_SCALE;
                if (post) { volatile float u = t * orc_h2f(post[b + i]); t = u; }
                y[(size_t)r * K + b + i] = orc_f2h(t);
            }
        }
}

/* ------------------------------------------------------------------------------------------------------------ */
/* Routing                                                                                                        */
/* ------------------------------------------------------------------------------------------------------------ */

/* Router logit of one (row, column) in this project's order: 32 lanes; lane l keeps 8 partial sums s_q (fp64, from
 * 0), adding to s_q the product x[j] * w[j] for j = 8 l + 256 i + q, i ascending; each product is formed in fp32 and
 * widened to fp64 (a bf16 x bf16 or fp16 x fp16 product has at most 22 significant bits, so it is exact unless it is
 * below 2^-126 or overflows fp32: only bf16 pairs far outside any model's range). The lane's value is
 * ((s0 + s1) + (s2 + s3)) + ((s4 + s5) + (s6 + s7)); the 32 lane values are combined by an xor tree over offsets
 * 16, 8, 4, 2, 1 (value of lane l becomes v_l + v_{l^o}), and lane 0's value is the logit. */
double orc_router_logit(const uint16_t* x, const uint16_t* w, int H) {
    double v[32];
    for (int l = 0; l < 32; ++l) {
        double s[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j0 = 8 * l; j0 < H; j0 += 256)
            for (int q = 0; q < 8; ++q) {
                const float pr = orc_bf2f(x[j0 + q]) * orc_bf2f(w[j0 + q]);
                s[q] = s[q] + (double)pr;
            }
        v[l] = ((s[0] + s[1]) + (s[2] + s[3])) + ((s[4] + s[5]) + (s[6] + s[7]));
    }
    for (int o = 16; o > 0; o >>= 1) {
        double t[32];
        for (int l = 0; l < 32; ++l) t[l] = v[l] + v[l ^ o];
        memcpy(v, t, sizeof(t));
    }
    return v[0];
}

/* Grouping (experts.cu:23-76): distinct experts < E in id order, members row * 32 + slot in (row, slot) order,
 * padded with -1 to maxm. Returns the distinct count. */
int orc_group(const int* pick, int R, int slots, int E, int* uids, int* members, int maxm, int maxu) {
    int cnt = 0;
    for (int e = 0; e < E; ++e) {
        int j = 0;
        for (int i = 0; i < R * slots; ++i)
            if (pick[i] == e) {
                if (j == 0) {
                    if (cnt >= maxu) return -1;
                    uids[cnt] = e;
                }
                if (j < maxm) members[cnt * maxm + j] = (i / slots) * 32 + (i % slots);
                ++j;
            }
        if (j) {
            for (int q = j; q < maxm; ++q) members[cnt * maxm + q] = -1;
            ++cnt;
        }
    }
    return cnt;
}

/* Fused routing (route.cu): logits (orc_router_logit) for E experts (+ the shared gate when sgate != NULL), each
 * expert logit rounded once to bf16; top-k by value with the lowest id on ties; weights = exp(l - lmax) over the
 * selected k, normalised (the full softmax denominator cancels in the reference's renormalisation); the shared slot
 * (id shared_id) gets sigmoid of its fp32 logit. x, gate, sgate: bf16 bits. Outputs pick/wts [R][k + has]. */
void orc_route(const uint16_t* x, int R, int H, const uint16_t* gate, int E, const uint16_t* sgate, int k,
               int shared_id, float* logits_bf, int* pick, float* wts) {
    const int has = sgate != NULL && shared_id >= 0;
    const int slots = k + has;
    for (int r = 0; r < R; ++r) {
        float* lb = logits_bf + (size_t)r * E;
        for (int e = 0; e < E; ++e) lb[e] = orc_bf2f(orc_d2bf(orc_router_logit(x + (size_t)r * H, gate + (size_t)e * H, H)));
        char* used = (char*)calloc((size_t)E, 1);
        int ids[64];
        for (int t = 0; t < k; ++t) {
            int be = -1;
            for (int e = 0; e < E; ++e)
                if (!used[e] && (be < 0 || lb[e] > lb[be])) be = e;
            used[be] = 1;
            ids[t] = be;
        }
        free(used);
        const float mx = lb[ids[0]];
        float p[64], sum = 0.f;
        for (int t = 0; t < k; ++t) { p[t] = expf(lb[ids[t]] - mx); sum += p[t]; }
        for (int t = 0; t < k; ++t) {
            pick[r * slots + t] = ids[t];
            wts[r * slots + t] = p[t] / sum;
        }
        if (has) {
            const float sl = (float)orc_router_logit(x + (size_t)r * H, sgate, H);
            pick[r * slots + k] = shared_id;
            wts[r * slots + k] = 1.0f / (1.0f + expf(-sl));
        }
    }
}

/* ------------------------------------------------------------------------------------------------------------ */
/* MoE expert pieces (experts.cu)                                                                                 */
/* ------------------------------------------------------------------------------------------------------------ */

/* Gate/up epilogue of one slot (experts.cu:120-162, act_mode 1 = fp32 SwiGLU, limit = inf):
 * g/u fp32 [N] raw sums -> xd fp16 [N] = fp16(FWHT(silu(FWHT(g)*HAD*svh_g) * FWHT(u)*HAD*svh_u * suh_d) * HAD) */
void orc_gateup_epilogue(const float* g, const float* u, int N, const uint16_t* svh_g, const uint16_t* svh_u,
                         const uint16_t* suh_d, uint16_t* xd) {
    for (int b = 0; b < N; b += 128) {
        float gv[128], uv[128], v[128];
        memcpy(gv, g + b, sizeof(gv));
        memcpy(uv, u + b, sizeof(uv));
        orc_fwht128(gv);
        orc_fwht128(uv);
        for (int i = 0; i < 128; ++i) {
            volatile float g1 = gv[i] * HAD_SCALE;
            volatile float gg = g1 * orc_h2f(svh_g[b + i]);
            volatile float u1 = uv[i] * HAD_SCALE;
            volatile float uu = u1 * orc_h2f(svh_u[b + i]);
            volatile float den = 1.f + expf(-gg);
            volatile float sg = gg / den;
            volatile float act = sg * uu;
            volatile float p = act * orc_h2f(suh_d[b + i]);
            v[i] = p;
        }
        orc_fwht128(v);
        for (int i = 0; i < 128; ++i) {
            volatile float t = v[i] * HAD_SCALE;
            xd[b + i] = orc_f2h(t);
        }
    }
}

/* Down epilogue of one slot (experts.cu:340-372): y fp32 [D] = FWHT(z) * HAD * svh_d, left to right. */
void orc_down_epilogue(const float* z, int D, const uint16_t* svh_d, float* y) {
    for (int b = 0; b < D; b += 128) {
        float v[128];
        memcpy(v, z + b, sizeof(v));
        orc_fwht128(v);
        for (int i = 0; i < 128; ++i) {
            volatile float t = v[i] * HAD_SCALE;
            volatile float o = t * orc_h2f(svh_d[b + i]);
            y[b + i] = o;
        }
    }
}

/* Combine one row (experts.cu:373-392): out = fma chain over the first n_routed slots from 0 in slot order. */
void orc_combine_row(const float* y, const float* w, int n_routed, int D, float* out) {
    for (int d = 0; d < D; ++d) {
        float acc = 0.f;
        for (int q = 0; q < n_routed; ++q) acc = fmaf(w[q], y[(size_t)q * D + d], acc);
        out[d] = acc;
    }
}
