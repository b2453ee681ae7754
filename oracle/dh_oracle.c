/*
 * dh_oracle.c -- CPU oracle for the MDLM sampler / output-head hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is a plain-C restatement of the
 * reference algorithms; it is the checker the CUDA path is compared against.
 * Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
 * arm may load it.  The product library never links or calls it.
 *
 * Parity is pinned against the reference itself: tests/test_oracle_pins.py
 * checks every function here against the Random123 known answers, the golden
 * factorized-Gumbel points, and against the reference HLS C++ compiled from
 * its own sources into oracle/_ref (see oracle/Makefile).
 *
 * Reference functions restated (paths inside K1ta141k/DiffusionHard):
 *   philox4x32_10            hls/rng/philox_rng.cpp:33-54, src/diffusion_accel/rng.py:36-61
 *   factorized Gumbel Q10    hls/rng/philox_rng.cpp:74-93, src/diffusion_accel/rng.py:111-193
 *   Gumbel tables            hls/rng/generate_gumbel_lut.py:14-33
 *   word stream order        hls/rng/philox_rng.cpp:95-149 (counter :137-139)
 *   requantize_q20           hls/output_head/output_head.cpp:10-19
 *   output head argmax       hls/output_head/output_head.cpp:23-157 (mask :138-140, strict > :147-151)
 *   candidate reveal         hls/candidate_sampler/candidate_sampler.cpp:5-79
 *   candidate-cache sampler  src/diffusion_accel/mdlm.py:1104-1218
 *   W8A8 dequant             src/diffusion_accel/fixed_mlp.py:65-136 (output :104-106)
 *   Q10 logits               src/diffusion_accel/rng.py:262
 *
 * Build: gcc -O2 -ffp-contract=off -fPIC -shared (oracle/Makefile).  No FMA
 * contraction: every float operation here is one IEEE operation.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_M0 0xD2511F53u
#define OR_M1 0xCD9E8D57u
#define OR_W0 0x9E3779B9u
#define OR_W1 0xBB67AE85u

/* ---------------------------------------------------------------- Philox */

void or_philox4x32_10(const uint32_t ctr_in[4], const uint32_t key_in[2],
                      uint32_t out[4]) {
    uint32_t c0 = ctr_in[0], c1 = ctr_in[1], c2 = ctr_in[2], c3 = ctr_in[3];
    uint32_t k0 = key_in[0], k1 = key_in[1];
    for (int round = 0; round < 10; ++round) {
        uint64_t p0 = (uint64_t)OR_M0 * c0;
        uint64_t p1 = (uint64_t)OR_M1 * c2;
        uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ k0;
        uint32_t n1 = (uint32_t)p1;
        uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ k1;
        uint32_t n3 = (uint32_t)p0;
        c0 = n0; c1 = n1; c2 = n2; c3 = n3;
        if (round != 9) {
            k0 += OR_W0;
            k1 += OR_W1;
        }
    }
    out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* Word for (token, position) in the reference stream layout: one Philox call
 * per group of 4 consecutive tokens, counter (token/4, position, eval, stream). */
uint32_t or_philox_token_word(uint32_t token, uint32_t position, uint32_t eval_id,
                              uint32_t stream_id, uint32_t key_lo, uint32_t key_hi) {
    uint32_t ctr[4] = {token >> 2, position, eval_id, stream_id};
    uint32_t key[2] = {key_lo, key_hi};
    uint32_t out[4];
    or_philox4x32_10(ctr, key, out);
    return out[token & 3u];
}

/* Reveal word: counter (position/4, 0, step, stream 1) -- build-defined layout
 * that keeps one word per (sequence, position, step). */
uint32_t or_reveal_word(uint32_t position, uint32_t step, uint32_t key_lo,
                        uint32_t key_hi) {
    uint32_t ctr[4] = {position >> 2, 0u, step, 1u};
    uint32_t key[2] = {key_lo, key_hi};
    uint32_t out[4];
    or_philox4x32_10(ctr, key, out);
    return out[position & 3u];
}

/* ----------------------------------------------------------- Gumbel Q10 */

static int16_t g_base[256];
static int16_t g_corr[3][256];
static int32_t g_top;
static int32_t g_log2q;
static int g_tables_ready;

static void or_init_tables(void) {
    if (g_tables_ready) return;
    const double scale = 1024.0;
    for (int m = 0; m < 256; ++m) {
        double mid = (256.0 + m + 0.5) / 256.0;
        g_base[m] = (int16_t)nearbyint(-log(mid) * scale);
        for (int e = 0; e < 3; ++e) {
            double u = mid * ldexp(1.0, -(e + 1));
            g_corr[e][m] = (int16_t)nearbyint(-log(-log1p(-u)) * scale);
        }
    }
    double top_u = 1.0 - 0.5 / 4294967296.0;
    g_top = (int32_t)nearbyint(-log(-log(top_u)) * scale);
    g_log2q = (int32_t)nearbyint(log(2.0) * scale);
    g_tables_ready = 1;
}

void or_gumbel_tables(int16_t base[256], int16_t corr[768], int32_t* top,
                      int32_t* log2q) {
    or_init_tables();
    memcpy(base, g_base, sizeof g_base);
    memcpy(corr, g_corr, sizeof g_corr);
    *top = g_top;
    *log2q = g_log2q;
}

static uint32_t or_clz32(uint32_t v) {
    uint32_t n = 0;
    if (v == 0) return 32;
    while (!(v & 0x80000000u)) { v <<= 1; ++n; }
    return n;
}

int32_t or_gumbel_q10(uint32_t word) {
    or_init_tables();
    uint32_t d = 0xFFFFFFFFu - word;
    if (d == 0) return g_top;
    uint32_t e = or_clz32(d);
    uint32_t fl = 31u - e;
    uint32_t norm = fl >= 8 ? (d >> (fl - 8)) : (d << (8 - fl));
    uint32_t m = norm - 256u;
    if (e < 3) return g_corr[e][m];
    return (int32_t)(e + 1) * g_log2q + g_base[m];
}

/* --------------------------------------------------------- Q10 logits */

/* round(logit * 1024) with round-half-to-even, as torch.round (rng.py:262).
 * Saturates to +-2^30 so that adding a Q10 Gumbel score cannot overflow. */
int32_t or_logit_q10(float logit) {
    float scaled = logit * 1024.0f;
    if (!(scaled == scaled)) return -(1 << 30);
    if (scaled > 1073741824.0f) return 1 << 30;
    if (scaled < -1073741824.0f) return -(1 << 30);
    return (int32_t)nearbyintf(scaled);
}

/* Noisy argmax over fp32 logits rows: score = Q10(logit) + Gumbel_Q10(word),
 * word from counter (token/4, row_position, row_eval, stream), key
 * (key_lo, row_key_hi).  Mask token skipped; strict '>' so the lowest id
 * wins ties (output_head.cpp:138-151). */
void or_noisy_argmax_f32(const float* logits, uint32_t rows, uint32_t vocab,
                         uint32_t mask_id, const uint32_t* row_position,
                         const uint32_t* row_key_hi, const uint32_t* row_eval,
                         uint32_t key_lo, uint32_t stream_id, int32_t* out_ids,
                         int32_t* out_scores) {
    for (uint32_t r = 0; r < rows; ++r) {
        const float* row = logits + (size_t)r * vocab;
        int64_t best = INT64_MIN;
        int32_t best_id = 0;
        uint32_t ctr[4] = {0, row_position[r], row_eval[r], stream_id};
        uint32_t key[2] = {key_lo, row_key_hi[r]};
        uint32_t words[4] = {0, 0, 0, 0};
        for (uint32_t v = 0; v < vocab; ++v) {
            if ((v & 3u) == 0) {
                ctr[0] = v >> 2;
                or_philox4x32_10(ctr, key, words);
            }
            if (v == mask_id) continue;
            int64_t s = (int64_t)or_logit_q10(row[v]) + or_gumbel_q10(words[v & 3u]);
            if (s > best) { best = s; best_id = (int32_t)v; }
        }
        out_ids[r] = best_id;
        if (out_scores) out_scores[r] = (int32_t)best;
    }
}

/* Greedy argmax over fp32 logits with the mask excluded, lowest id on ties
 * (mdlm.py:1190-1191 on logits; torch.argmax returns the first maximum). */
void or_greedy_argmax_f32(const float* logits, uint32_t rows, uint32_t vocab,
                          uint32_t mask_id, int32_t* out_ids) {
    for (uint32_t r = 0; r < rows; ++r) {
        const float* row = logits + (size_t)r * vocab;
        float best = -INFINITY;
        int32_t best_id = -1;
        for (uint32_t v = 0; v < vocab; ++v) {
            if (v == mask_id) continue;
            if (best_id < 0 || row[v] > best) { best = row[v]; best_id = (int32_t)v; }
        }
        out_ids[r] = best_id < 0 ? 0 : best_id;
    }
}

/* ------------------------------------------------------ int8 output head */

int32_t or_requantize_q20(int32_t acc, int32_t mult_q20) {
    int64_t prod = (int64_t)acc * mult_q20;
    const int64_t half = (int64_t)1 << 19;
    if (prod >= 0) return (int32_t)((prod + half) >> 20);
    return -(int32_t)((-prod + half) >> 20);
}

static int32_t or_dot_i8(const int8_t* a, const int8_t* b, uint32_t n) {
    int32_t acc = 0;
    for (uint32_t k = 0; k < n; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
    return acc;
}

/* int32 accumulators of A[rows,k] x W[n,k]^T (the int8 tensor-engine contract). */
void or_gemm_i8(const int8_t* a, const int8_t* w, uint32_t rows, uint32_t n,
                uint32_t k, int32_t* out) {
    for (uint32_t r = 0; r < rows; ++r)
        for (uint32_t j = 0; j < n; ++j)
            out[(size_t)r * n + j] = or_dot_i8(a + (size_t)r * k, w + (size_t)j * k, k);
}

/* The model-path logit of one head element, bit-identical to the reference's
 * W8A8 linear (fixed_mlp.py:98-106):  combined = a_scale * w_scale (fp32),
 * out = float(double(acc) * double(combined) + double(bias)). */
float or_dequant_logit(int32_t acc, float a_scale, float w_scale, float bias) {
    float combined = a_scale * w_scale;
    double v = (double)acc * (double)combined + (double)bias;
    return (float)v;
}

/* Head modes. */
enum { OR_HEAD_REQUANT_Q20 = 0, OR_HEAD_DEQUANT_NOISY = 1, OR_HEAD_DEQUANT_GREEDY = 2 };

/*
 * Fused int8 head + noisy argmax.
 *   mode REQUANT_Q20: HLS contract, score = requant(acc, mult_q20[v]) +
 *       bias_q10[v] + noise (output_head.cpp:141-146).  `noise` (rows x vocab,
 *       row-major) is used when non-NULL, else the Philox-Gumbel word of
 *       (v, row_position[r], row_eval[r], stream) with key (key_lo, row_key_hi[r]).
 *   mode DEQUANT_NOISY: score = Q10(dequant logit) + Gumbel.
 *   mode DEQUANT_GREEDY: argmax of the fp32 dequant logit.
 * Mask skipped, lowest id on ties.  out_scores (optional) receives the
 * winning integer score (modes 0/1) or the float bits of the winning logit (2).
 */
void or_head_i8(int mode, const int8_t* hidden, const int8_t* weights,
                uint32_t rows, uint32_t hidden_size, uint32_t vocab,
                uint32_t mask_id, const int32_t* mult_q20, const int32_t* bias_q10,
                const int32_t* noise, const float* a_scale, const float* w_scale,
                const float* bias, const uint32_t* row_position,
                const uint32_t* row_key_hi, const uint32_t* row_eval,
                uint32_t key_lo, uint32_t stream_id, int32_t* out_ids,
                int32_t* out_scores) {
    for (uint32_t r = 0; r < rows; ++r) {
        const int8_t* h = hidden + (size_t)r * hidden_size;
        int64_t best = INT64_MIN;
        float bestf = -INFINITY;
        int32_t best_id = -1;
        uint32_t ctr[4] = {0, row_position ? row_position[r] : r,
                           row_eval ? row_eval[r] : 0, stream_id};
        uint32_t key[2] = {key_lo, row_key_hi ? row_key_hi[r] : 0};
        uint32_t words[4] = {0, 0, 0, 0};
        for (uint32_t v = 0; v < vocab; ++v) {
            if (mode != OR_HEAD_DEQUANT_GREEDY && (v & 3u) == 0 && !noise) {
                ctr[0] = v >> 2;
                or_philox4x32_10(ctr, key, words);
            }
            if (v == mask_id) continue;
            int32_t acc = or_dot_i8(h, weights + (size_t)v * hidden_size, hidden_size);
            if (mode == OR_HEAD_DEQUANT_GREEDY) {
                float l = or_dequant_logit(acc, a_scale[r], w_scale[v], bias[v]);
                if (best_id < 0 || l > bestf) { bestf = l; best_id = (int32_t)v; }
                continue;
            }
            int32_t g = noise ? noise[(size_t)r * vocab + v] : or_gumbel_q10(words[v & 3u]);
            int64_t s;
            if (mode == OR_HEAD_REQUANT_Q20)
                s = (int64_t)or_requantize_q20(acc, mult_q20[v]) + bias_q10[v] + g;
            else
                s = (int64_t)or_logit_q10(or_dequant_logit(acc, a_scale[r], w_scale[v], bias[v])) + g;
            if (s > best) { best = s; best_id = (int32_t)v; }
        }
        out_ids[r] = best_id < 0 ? 0 : best_id;
        if (out_scores) {
            if (mode == OR_HEAD_DEQUANT_GREEDY) memcpy(&out_scores[r], &bestf, 4);
            else out_scores[r] = (int32_t)best;
        }
    }
}

/* --------------------------------------------------- candidate reveal */

/* candidate_sampler.cpp:5-79 without the 256-position cap: the invalidation
 * on any change clears the valid bits of the whole sequence. Returns
 * (status << 32) | changed; status 1 = bad position count, 2 = threshold > 2^32.
 * No state is touched on error. */
uint64_t or_candidate_reveal(uint16_t* tokens, const uint16_t* cands,
                             uint64_t* active, uint64_t* valid,
                             const uint32_t* words, uint64_t threshold_q32,
                             uint32_t positions) {
    if (positions == 0) return (uint64_t)1 << 32;
    if (threshold_q32 > ((uint64_t)1 << 32)) return (uint64_t)2 << 32;
    uint32_t changed = 0;
    for (uint32_t p = 0; p < positions; ++p) {
        uint64_t bit = (uint64_t)1 << (p & 63);
        uint32_t w = p >> 6;
        int a = (active[w] & bit) != 0;
        int v = (valid[w] & bit) != 0;
        int reveal = (uint64_t)words[p] < threshold_q32;
        if (a && v && reveal) {
            tokens[p] = cands[p];
            active[w] &= ~bit;
            ++changed;
        }
    }
    if (changed) {
        for (uint32_t w = 0; w < (positions + 63) / 64; ++w) valid[w] = 0;
    }
    return changed;
}

/* ------------------------------------------- candidate-cache sampler loop */

/*
 * Candidate-cache DDPM loop over fp32 logits supplied by a fake model
 * (mdlm.py:1104-1218 with the counter-based RNG).  One sequence per call.
 *   logits_per_eval: (steps + 1) blocks of [positions, vocab]; block k is what
 *       the model returns when it is evaluated at transition k, block `steps`
 *       is the final greedy pass.
 *   thr_q32[steps]: reveal thresholds (floor(p_k * 2^32), capped at 2^32).
 *   key = (seed, seq_index); noise counter (v/4, p, k, 0); reveal word
 *       counter (p/4, 0, k, 1).
 * Outputs: tokens (in/out), per-step snapshots of tokens / candidates /
 * active / valid bitmaps (optional, may be NULL), per-step active and changed
 * counts, evaluated flags; returns the number of model evaluations.
 */
uint32_t or_candidate_cache_sampler_f32(
    const float* logits_per_eval, uint32_t positions, uint32_t vocab,
    uint32_t mask_id, uint32_t steps, const uint64_t* thr_q32, uint32_t seed,
    uint32_t seq_index, int32_t* tokens, int32_t* snap_tokens,
    int32_t* snap_cands, uint64_t* snap_active, uint64_t* snap_valid,
    int32_t* step_active, int32_t* step_changed, int32_t* step_evaluated,
    uint32_t* transitions_out) {
    uint32_t words_n = (positions + 63) / 64;
    uint16_t* tok16 = (uint16_t*)calloc(positions, 2);
    uint16_t* cand16 = (uint16_t*)calloc(positions, 2);
    uint64_t* active = (uint64_t*)calloc(words_n, 8);
    uint64_t* valid = (uint64_t*)calloc(words_n, 8);
    uint32_t* rw = (uint32_t*)calloc(positions, 4);
    uint32_t* pos = (uint32_t*)calloc(positions, 4);
    uint32_t* khi = (uint32_t*)calloc(positions, 4);
    uint32_t* ev = (uint32_t*)calloc(positions, 4);
    int32_t* ids = (int32_t*)calloc(positions, 4);
    uint32_t evaluations = 0, transitions = 0;
    for (uint32_t p = 0; p < positions; ++p) {
        tok16[p] = (uint16_t)tokens[p];
        if ((uint32_t)tokens[p] == mask_id) active[p >> 6] |= (uint64_t)1 << (p & 63);
        pos[p] = p;
        khi[p] = seq_index;
    }
    for (uint32_t k = 0; k < steps; ++k) {
        uint32_t active_count = 0;
        for (uint32_t w = 0; w < words_n; ++w) active_count += (uint32_t)__builtin_popcountll(active[w]);
        if (active_count == 0) break;
        ++transitions;
        step_active[k] = (int32_t)active_count;
        int cache_valid = 0;
        for (uint32_t w = 0; w < words_n; ++w) cache_valid |= valid[w] != 0;
        step_evaluated[k] = !cache_valid;
        if (!cache_valid) {
            for (uint32_t p = 0; p < positions; ++p) ev[p] = k;
            or_noisy_argmax_f32(logits_per_eval + (size_t)k * positions * vocab,
                                positions, vocab, mask_id, pos, khi, ev, seed, 0u,
                                ids, NULL);
            for (uint32_t p = 0; p < positions; ++p) {
                cand16[p] = (uint16_t)ids[p];
                valid[p >> 6] |= (uint64_t)1 << (p & 63);
            }
            ++evaluations;
        }
        for (uint32_t p = 0; p < positions; ++p) rw[p] = or_reveal_word(p, k, seed, seq_index);
        uint64_t res = or_candidate_reveal(tok16, cand16, active, valid, rw, thr_q32[k], positions);
        step_changed[k] = (int32_t)(uint32_t)res;
        if (snap_tokens) for (uint32_t p = 0; p < positions; ++p) snap_tokens[(size_t)k * positions + p] = tok16[p];
        if (snap_cands) for (uint32_t p = 0; p < positions; ++p) snap_cands[(size_t)k * positions + p] = cand16[p];
        if (snap_active) memcpy(snap_active + (size_t)k * words_n, active, words_n * 8);
        if (snap_valid) memcpy(snap_valid + (size_t)k * words_n, valid, words_n * 8);
    }
    uint32_t remaining = 0;
    for (uint32_t w = 0; w < words_n; ++w) remaining += (uint32_t)__builtin_popcountll(active[w]);
    if (remaining) {
        or_greedy_argmax_f32(logits_per_eval + (size_t)steps * positions * vocab, positions,
                             vocab, mask_id, ids);
        for (uint32_t p = 0; p < positions; ++p)
            if (active[p >> 6] & ((uint64_t)1 << (p & 63))) tok16[p] = (uint16_t)ids[p];
        ++evaluations;
    }
    for (uint32_t p = 0; p < positions; ++p) tokens[p] = tok16[p];
    if (transitions_out) *transitions_out = transitions;
    free(tok16); free(cand16); free(active); free(valid); free(rw); free(pos);
    free(khi); free(ev); free(ids);
    return evaluations;
}
