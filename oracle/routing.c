/*
 * ORACLE — test infrastructure only.  Nothing in the product links or calls this file; only
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference arm load it, as the
 * checker.
 *
 * CPU restatement of the router of the MoE block, written to the same fixed arithmetic order
 * that the CUDA router kernel uses, so that logits, probabilities and expert choices compare
 * bit for bit.  The reference computes:
 *
 *   Switch (src/harmonymoe/router.py:52-63, Router.standard_forward):
 *     logits = Linear(x)              in the router-weight dtype tau (router.py:37-45)
 *     probs  = softmax(logits)        in tau
 *     e      = argmax(probs)          first index on ties
 *     g      = max(probs)             in tau
 *   Qwen (qwen_ep_adapter/qwen_ep.py:48-53, ShardedQwenMoE.forward):
 *     logits = gate(x)                bf16
 *     probs  = softmax(logits, dtype=float32)
 *     (w, c) = topk(probs, k)         ties: probability descending, expert id ascending
 *     w      = w / sum(w)             only when norm_topk_prob
 *     w      = w.to(activation dtype)
 *
 * Fixed order used here and in the kernels (the reference leaves it to cuBLAS/ATen); the
 * optional tensor-core router follows oracle_router_logits_fixed instead:
 *   C          = 32 * ceil(d / 256)   (d splits into at most 8 chunks of C)
 *   S_q        = fma-accumulate over i in [qC, min(d, (q+1)C)) of x[t,i] * W[e,i], from 0.0f
 *   logit[t,e] = round_tau( partials summed left to right: ((S_0 + S_1) + S_2) + ... )
 *   m          = max_e logit[t,e]
 *   ex[e]      = dsca_exp(logit[t,e] - m)
 *   s          = 32 lane partials (lane L sums e = L, L+32, L+64 ... in that order) combined by
 *                the xor butterfly 16, 8, 4, 2, 1
 *   p[e]       = ex[e] / s          (IEEE division)
 * dsca_exp is a Cody-Waite reduction (x = n ln2 + r, ln2 split in a 16-bit head and a tail)
 * followed by the degree-7 Taylor polynomial of e^r in Horner form, scaled by 2^n through the
 * exponent bits; inputs below -87 give 0.  Every step is an IEEE-754 single operation, so the
 * C and CUDA versions return the same bits.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off; fmaf is the correctly rounded libm fmaf).
 */
#include <math.h>
#include <stdlib.h>
#include <stdint.h>
#include <string.h>

static float bits_to_f(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }
static uint32_t f_to_bits(float f) { uint32_t u; memcpy(&u, &f, 4); return u; }

/* round-to-nearest-even to bfloat16, returned as float */
float oracle_round_bf16(float f) {
    uint32_t u = f_to_bits(f);
    if ((u & 0x7f800000u) == 0x7f800000u) {          /* inf / nan pass through */
        if (u & 0x007fffffu) u |= 0x00400000u;
        return bits_to_f(u & 0xffff0000u);
    }
    uint32_t lsb = (u >> 16) & 1u;
    u = u + 0x7fffu + lsb;
    return bits_to_f(u & 0xffff0000u);
}

/* e^x for x <= 0 (larger x is clamped to 0) */
float oracle_exp_neg(float x) {
    if (!(x <= 0.0f)) x = 0.0f;
    if (x < -87.0f) return 0.0f;
    const float log2e = 1.44269504088896341f;
    const float ln2_hi = 0.693145751953125f;       /* 16 significant bits: n*ln2_hi is exact */
    const float ln2_lo = 1.42860682030941723e-6f;  /* ln 2 - ln2_hi */
    float n = rintf(x * log2e);
    float r = fmaf(-n, ln2_hi, x);
    r = fmaf(-n, ln2_lo, r);
    float p = 1.0f / 5040.0f;
    p = fmaf(p, r, 1.0f / 720.0f);
    p = fmaf(p, r, 1.0f / 120.0f);
    p = fmaf(p, r, 1.0f / 24.0f);
    p = fmaf(p, r, 1.0f / 6.0f);
    p = fmaf(p, r, 0.5f);
    p = fmaf(p, r, 1.0f);
    p = fmaf(p, r, 1.0f);
    int ni = (int)n;                                /* -126 <= ni <= 0 */
    float scale = bits_to_f((uint32_t)(ni + 127) << 23);
    return p * scale;
}

/* Chunk length of the logit sum: C = 32 * ceil(d / 256), so d splits into at most 8 chunks. */
int oracle_router_chunk(int d) { return 32 * ((d + 255) / 256); }

/*
 * logits[T,E] = round_tau(x[T,d] . W[E,d]^T); round_bf16 selects tau = bf16, else fp32.
 * Order: chunk q covers i in [qC, min(d, (q+1)C)); its partial S_q is the fma chain over i in
 * increasing order from 0.0f; the logit is (((S_0 + S_1) + S_2) + ...) + S_7, left to right.
 */
void oracle_router_logits(const float* x, const float* W, int T, int d, int E, int round_bf16,
                          float* logits) {
    const int C = oracle_router_chunk(d);
    for (int t = 0; t < T; ++t) {
        const float* xr = x + (size_t)t * d;
        for (int e = 0; e < E; ++e) {
            const float* wr = W + (size_t)e * d;
            float acc = 0.0f;
            for (int q = 0; q * C < d; ++q) {
                const int i1 = (q + 1) * C < d ? (q + 1) * C : d;
                float s = 0.0f;
                for (int i = q * C; i < i1; ++i) s = fmaf(xr[i], wr[i], s);
                acc = (q == 0) ? s : acc + s;
            }
            logits[(size_t)t * E + e] = round_bf16 ? oracle_round_bf16(acc) : acc;
        }
    }
}



/*
 * bf16 logits by exact fixed-point accumulation (the arithmetic of the tensor-core router).
 * A bf16 value v (sign s, biased exponent b, 7-bit mantissa m) is s * M * 2^(e - 134) with
 * M = 128 + m, e = b for normals and M = m, e = 1 for zero and subnormals.  With R the largest e
 * over the row's nonzero entries (1 for an all-zero row), v is held as the 21-bit magnitude
 *   F = M << (13 - (R - e))        when R - e <= 13  (exact: v = s F 2^(R - 147)),
 *   F = M >> ((R - e) - 13)        otherwise          (low bits dropped; 0 from R - e = 21 on),
 * and the logit of (x row, W row) is
 *   P        = sum_i s_x s_w F_x F_w                 exact, in a 64-bit integer
 *   logit32  = (float) P                             round to nearest even
 *   logit32  = logit32 * 2^(R_x + R_w - 294)         IEEE multiplications by powers of two
 *   logit    = round_bf16(logit32).
 * The device splits each F into three signed 7-bit slices and accumulates the nine slice
 * products in 32-bit integers on the tensor cores; the integer sum is the same P.
 * Inputs are bf16 values carried in floats; non-finite inputs are not supported.
 */
static void fixed_row(const float* v, int d, int32_t* F, int* R) {
    int rmax = 1;
    for (int i = 0; i < d; ++i) {
        const uint32_t u = f_to_bits(v[i]) >> 16;
        const int b = (int)((u >> 7) & 0xffu);
        const int m = (int)(u & 0x7fu);
        if ((b != 0 || m != 0) && b > rmax) rmax = b;
    }
    for (int i = 0; i < d; ++i) {
        const uint32_t u = f_to_bits(v[i]) >> 16;
        const int b = (int)((u >> 7) & 0xffu);
        const int m = (int)(u & 0x7fu);
        const int M = b ? 128 + m : m;
        const int e = b ? b : 1;
        const int sh = rmax - e;
        int32_t f = sh <= 13 ? (M << (13 - sh)) : (sh - 13 < 9 ? (M >> (sh - 13)) : 0);
        F[i] = (u & 0x8000u) ? -f : f;
    }
    *R = rmax;
}

/* f * 2^k by IEEE single multiplications, each factor a normal power of two */
float oracle_scale_pow2(float f, int k) {
    while (k > 127) { f = f * bits_to_f(254u << 23); k -= 127; }
    while (k < -126) { f = f * bits_to_f(1u << 23); k += 126; }
    return f * bits_to_f((uint32_t)(k + 127) << 23);
}

void oracle_router_logits_fixed(const float* x, const float* W, int T, int d, int E, float* logits) {
    int32_t* fw = (int32_t*)malloc(sizeof(int32_t) * (size_t)E * d);
    int* rw = (int*)malloc(sizeof(int) * (size_t)E);
    int32_t* fx = (int32_t*)malloc(sizeof(int32_t) * (size_t)d);
    for (int e = 0; e < E; ++e) fixed_row(W + (size_t)e * d, d, fw + (size_t)e * d, rw + e);
    for (int t = 0; t < T; ++t) {
        int rx;
        fixed_row(x + (size_t)t * d, d, fx, &rx);
        for (int e = 0; e < E; ++e) {
            const int32_t* w = fw + (size_t)e * d;
            int64_t p = 0;
            for (int i = 0; i < d; ++i) p += (int64_t)fx[i] * (int64_t)w[i];
            const float l = oracle_scale_pow2((float)p, rx + rw[e] - 294);
            logits[(size_t)t * E + e] = oracle_round_bf16(l);
        }
    }
    free(fw);
    free(rw);
    free(fx);
}

/* softmax of one row in the kernel's order; probs[E] fp32 (not rounded) */
static void softmax_row(const float* l, int E, float* probs) {
    float m = l[0];
    for (int e = 1; e < E; ++e) m = (l[e] > m) ? l[e] : m;
    float part[32];
    for (int L = 0; L < 32; ++L) {
        float s = 0.0f;
        for (int e = L; e < E; e += 32) s = s + oracle_exp_neg(l[e] - m);
        part[L] = s;
    }
    for (int off = 16; off >= 1; off >>= 1) {
        float nxt[32];
        for (int L = 0; L < 32; ++L) nxt[L] = part[L] + part[L ^ off];
        memcpy(part, nxt, sizeof(part));
    }
    float s = part[0];
    for (int e = 0; e < E; ++e) probs[e] = oracle_exp_neg(l[e] - m) / s;
}

/*
 * Top-1 Switch routing.  logits hold tau values.  probs_round_bf16 rounds the probabilities to
 * bf16 before the argmax (tau = bf16).  Outputs: idx[T], gate[T] (the tau-rounded max prob).
 */
void oracle_route_top1(const float* logits, int T, int E, int probs_round_bf16, int32_t* idx,
                       float* gate) {
    float probs[1024];
    for (int t = 0; t < T; ++t) {
        softmax_row(logits + (size_t)t * E, E, probs);
        int best = 0;
        float bv = probs_round_bf16 ? oracle_round_bf16(probs[0]) : probs[0];
        for (int e = 1; e < E; ++e) {
            float v = probs_round_bf16 ? oracle_round_bf16(probs[e]) : probs[e];
            if (v > bv) { bv = v; best = e; }
        }
        idx[t] = best;
        gate[t] = bv;
    }
}

/*
 * Top-k Qwen routing over fp32 probabilities: ranking (p desc, id asc).  norm_topk divides by
 * the sum of the k chosen probabilities (summed in rank order); w_round_bf16 rounds the
 * weights to bf16 (activation dtype bf16).  Outputs ids[T,k], w[T,k].
 */
void oracle_route_topk(const float* logits, int T, int E, int k, int norm_topk, int w_round_bf16,
                       int32_t* ids, float* w) {
    float probs[1024];
    int taken[1024];
    for (int t = 0; t < T; ++t) {
        softmax_row(logits + (size_t)t * E, E, probs);
        for (int e = 0; e < E; ++e) taken[e] = 0;
        float sel[64];
        for (int j = 0; j < k; ++j) {
            int best = -1;
            for (int e = 0; e < E; ++e) {
                if (taken[e]) continue;
                if (best < 0 || probs[e] > probs[best]) best = e;
            }
            taken[best] = 1;
            ids[(size_t)t * k + j] = best;
            sel[j] = probs[best];
        }
        float sum = 0.0f;
        if (norm_topk)
            for (int j = 0; j < k; ++j) sum = sum + sel[j];
        for (int j = 0; j < k; ++j) {
            float v = norm_topk ? sel[j] / sum : sel[j];
            w[(size_t)t * k + j] = w_round_bf16 ? oracle_round_bf16(v) : v;
        }
    }
}

/* full probability rows (for diagnostics and near-tie classification) */
void oracle_softmax(const float* logits, int T, int E, float* probs) {
    for (int t = 0; t < T; ++t) softmax_row(logits + (size_t)t * E, E, probs + (size_t)t * E);
}

/* oracle_exp_neg over an array (test helper) */
void oracle_exp_neg_array(const float* x, float* y, long n) {
    for (long i = 0; i < n; ++i) y[i] = oracle_exp_neg(x[i]);
}
