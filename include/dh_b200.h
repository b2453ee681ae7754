/*
 * dh_b200.h -- C ABI of libdh_b200.so, the B200 (sm_100a) implementation of
 * the MDLM denoising hot path of K1ta141k/DiffusionHard.
 *
 * Conventions (mirroring the reference HLS kernels, hls/rng/philox_rng.hpp:29-33,
 * hls/output_head/output_head.hpp:20-26, hls/candidate_sampler/candidate_sampler.hpp:18-29):
 *   - every entry point returns a uint32_t status (0 = OK) and validates its
 *     arguments BEFORE touching any buffer; a non-zero status means nothing was
 *     launched and no output was written;
 *   - entry points that mirror a reference function return that function's own
 *     status codes (listed per family below); generic failures use codes >= 100;
 *   - all array arguments are DEVICE pointers owned by the caller; no entry
 *     point allocates memory.  Scratch space is passed as `workspace` whose
 *     size the matching *_workspace_size() query returns;
 *   - work is enqueued on the given CUDA stream (`void*` = cudaStream_t; NULL =
 *     legacy default stream) and is asynchronous; entry points are stateless
 *     and reentrant for distinct buffers / streams;
 *   - randomness is counter-based (Philox4x32-10), so no RNG state is held.
 *
 * Counter layouts (build-defined where the reference leaves them open):
 *   noise word for token v of a row:  philox((v/4, position, eval_id, stream_id),
 *                                            (key_lo, key_hi))[v % 4]
 *       -- identical to the reference stream kernels, philox_rng.cpp:137-139;
 *   reveal word of a position:        philox((position/4, 0, step, 1),
 *                                            (seed, sequence))[position % 4].
 */
#ifndef DH_B200_H
#define DH_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------ status codes */

/* Generic codes shared by every entry point. */
#define DH_OK 0u
#define DH_ERR_NULL_POINTER 100u
#define DH_ERR_ALIGNMENT 101u
#define DH_ERR_WORKSPACE 102u
#define DH_ERR_UNSUPPORTED_SHAPE 103u
#define DH_ERR_CUDA 104u
#define DH_ERR_INVALID_ARGUMENT 105u
#define DH_ERR_SCRATCH_LIMIT 106u
#define DH_ERR_NCCL 107u

/* RNG family -- same values as RngKernelStatus (philox_rng.hpp:29-33). */
#define DH_RNG_INVALID_POSITION_COUNT 1u
#define DH_RNG_INVALID_VOCABULARY_SIZE 2u

/* Output-head family -- same values as OutputHeadKernelStatus (output_head.hpp:20-26). */
#define DH_HEAD_INVALID_POSITION_COUNT 1u
#define DH_HEAD_INVALID_HIDDEN_SIZE 2u
#define DH_HEAD_INVALID_VOCABULARY_SIZE 3u
#define DH_HEAD_INVALID_MASK_TOKEN 4u

/* Candidate family -- same values as CandidateKernelStatus (candidate_sampler.hpp:12-16). */
#define DH_CAND_INVALID_POSITION_COUNT 1u
#define DH_CAND_INVALID_THRESHOLD 2u

/* Reveal probability one in Q32 (candidate_sampler.hpp:10). */
#define DH_REVEAL_PROBABILITY_ONE_Q32 (((uint64_t)1) << 32)

/* ------------------------------------------------------------------- RNG */

/* Philox4x32-10 on `count` independent (counter[4], key[2]) pairs; out[4*i..].
 * Replaces philox4x32_10, hls/rng/philox_rng.cpp:33-54 / rng.py:36-61. */
uint32_t dh_philox4x32_10(const uint32_t* counters, const uint32_t* keys, uint32_t* out,
                          uint32_t count, void* stream);

/* Factorized Q5.10 Gumbel score of each word.
 * Replaces factorized_gumbel_score_q10, hls/rng/philox_rng.cpp:74-93. */
uint32_t dh_gumbel_q10(const uint32_t* words, int32_t* scores, uint32_t count, void* stream);

/* Word / score streams in the reference order (vocab tiles of 16, then
 * position, then lane blocks of 4); `out` holds position_count*vocabulary_size
 * entries.  Limits and status codes as the reference: 1 <= positions <= 64,
 * 1 <= vocabulary <= 65535.
 * Replace philox_word_stream_kernel (philox_rng.cpp:95-149) and
 * philox_gumbel_stream_kernel (philox_rng.cpp:151-205). */
uint32_t dh_philox_word_stream(uint32_t* out, uint32_t position_count,
                               uint32_t vocabulary_size, uint32_t evaluation_id,
                               uint32_t stream_id, uint32_t seed_low, uint32_t seed_high,
                               void* stream);
uint32_t dh_philox_gumbel_stream(int32_t* out, uint32_t position_count,
                                 uint32_t vocabulary_size, uint32_t evaluation_id,
                                 uint32_t stream_id, uint32_t seed_low, uint32_t seed_high,
                                 void* stream);

/* ------------------------------------------------- noisy argmax over logits */

/* Gumbel-max candidate per row of fp32 logits (K1):
 *   score(v) = round_half_even(logit[v] * 1024) + gumbel_q10(word(v)),
 *   word(v) = philox((v/4, row_position[r], row_eval[r], stream_id),
 *                    (key_lo, row_key_hi[r]))[v%4];
 * the mask token is skipped and the lowest id wins ties.  Replaces the
 * exponential race of mdlm._sample_categorical (mdlm.py:844-849) with the
 * reference's hardware Q10 Gumbel race (rng.py:262-263, output_head.cpp:147-151).
 * row_position / row_key_hi / row_eval may be NULL (= row index / 0 / 0).
 * out_scores may be NULL.  Status: RNG family codes (rows == 0 ->
 * DH_RNG_INVALID_POSITION_COUNT, vocab == 0 or > 65535 or mask >= vocab ->
 * DH_RNG_INVALID_VOCABULARY_SIZE), DH_ERR_* otherwise. */
size_t dh_noisy_argmax_workspace_size(uint32_t rows, uint32_t vocabulary_size);
uint32_t dh_noisy_argmax_f32(const float* logits, uint64_t row_stride, uint32_t rows,
                             uint32_t vocabulary_size, uint32_t mask_token_id,
                             const uint32_t* row_position, const uint32_t* row_key_hi,
                             const uint32_t* row_eval, uint32_t key_lo, uint32_t stream_id,
                             int32_t* out_ids, int32_t* out_scores, void* workspace,
                             size_t workspace_bytes, void* stream);

/* dh_noisy_argmax_f32 for callers that cannot allocate device memory, such
 * as a plugin running inside a host framework that owns every device
 * allocation, or code that must not call cudaMalloc (which may synchronise
 * the device) once serving has started.  No counterpart in the reference.
 * Same arguments, results and status codes, minus the workspace: the
 * scratch is a 512 KiB array inside the library (held by every GPU that loads
 * it until the process exits).  rows * ceil(vocabulary_size / 4096) must not
 * exceed 65,536 (e.g. 5,041 rows of the 50,258-token vocabulary), else
 * DH_ERR_SCRATCH_LIMIT.  The first call on a device looks up the array's
 * device address (cudaGetSymbolAddress), so make that first call before any
 * stream capture; after a device reset the first call in the new context
 * looks it up again.  Calls share the array: calls that overlap on one GPU
 * race and must be serialised by the caller.  Allocates nothing. */
uint32_t dh_noisy_argmax_f32_noalloc(const float* logits, uint64_t row_stride, uint32_t rows,
                                     uint32_t vocabulary_size, uint32_t mask_token_id,
                                     const uint32_t* row_position, const uint32_t* row_key_hi,
                                     const uint32_t* row_eval, uint32_t key_lo, uint32_t stream_id,
                                     int32_t* out_ids, int32_t* out_scores, void* stream);

/* Greedy argmax of fp32 logits (mask skipped, lowest id on ties): the final
 * pass of the samplers, mdlm.py:1177-1200.  Same workspace as above. */
uint32_t dh_greedy_argmax_f32(const float* logits, uint64_t row_stride, uint32_t rows,
                              uint32_t vocabulary_size, uint32_t mask_token_id,
                              int32_t* out_ids, void* workspace, size_t workspace_bytes,
                              void* stream);

/* ----------------------------------------------------- candidate reveal (K2) */

/* Batched form of candidate_reveal_kernel (candidate_sampler.cpp:5-79) over
 * `sequences` independent canvases of `positions` each (no 256 cap): per
 * sequence, every position with active & valid & (word < threshold_q32)
 * takes its candidate and clears its active bit; if any position of the
 * sequence changed, ALL valid bits of that sequence are cleared.
 * Layouts: tokens / candidates / words [sequences][positions]; bitmaps
 * [sequences][ceil(positions/64)].  results[s] = (status << 32) | changed.
 * Status: DH_CAND_INVALID_POSITION_COUNT (positions == 0),
 * DH_CAND_INVALID_THRESHOLD (threshold > 2^32). */
uint32_t dh_candidate_reveal(uint16_t* tokens, const uint16_t* candidates, uint64_t* active,
                             uint64_t* valid, const uint32_t* words, uint64_t threshold_q32,
                             uint32_t positions, uint32_t sequences, uint64_t* results,
                             void* stream);

/* ------------------------------------------ candidate-cache sampler (device) */

/*
 * Device-resident state of the candidate-cache DDPM loop (mdlm.py:1104-1218)
 * for B sequences of L positions:
 *   tokens      int32  [B*L]   canvas (mask id = masked)
 *   candidates  uint16 [B*L]   cached candidate per position
 *   active      uint64 [B*W]   bit = position still masked        (W = ceil(L/64))
 *   valid       uint64 [B*W]   bit = cached candidate valid
 *   eval_id     uint32 [B]     transition index of the last model evaluation
 *   counters    int32  [3*steps]  per transition: batch active count, changed
 *                              count, 1 if any sequence evaluated (else 0)
 * Per sequence the cache is refilled when it is empty (the reference clears
 * the whole cache on any change, mdlm.py:1173-1174).
 */
uint32_t dh_sampler_init(const int32_t* input_ids, uint32_t sequences, uint32_t positions,
                         uint32_t mask_token_id, uint32_t steps, int32_t* tokens,
                         uint16_t* candidates, uint64_t* active, uint64_t* valid,
                         uint32_t* eval_id, int32_t* counters, void* stream);

/* One transition over externally supplied fp32 logits [B*L, vocab] (the
 * model(input_ids) / logits_function protocol): refill the candidate cache
 * of every sequence whose cache is empty and that still has masked positions
 * (K1 over its rows), then reveal with threshold_q32 (K2 with in-kernel
 * reveal words).  `logits` is only read for sequences that refill. */
size_t dh_sampler_workspace_size(uint32_t sequences, uint32_t positions,
                                 uint32_t vocabulary_size);
uint32_t dh_sampler_transition_f32(const float* logits, uint32_t sequences, uint32_t positions,
                                   uint32_t vocabulary_size, uint32_t mask_token_id,
                                   uint32_t seed, uint32_t step, uint32_t steps,
                                   uint64_t threshold_q32, int32_t* tokens,
                                   uint16_t* candidates, uint64_t* active, uint64_t* valid,
                                   uint32_t* eval_id, int32_t* counters, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Final greedy pass: every still-masked position takes the argmax of its
 * fp32 logits row (mask skipped, lowest id on ties), mdlm.py:1177-1200. */
uint32_t dh_sampler_finalize_f32(const float* logits, uint32_t sequences, uint32_t positions,
                                 uint32_t vocabulary_size, uint32_t mask_token_id,
                                 int32_t* tokens, uint64_t* active, void* workspace,
                                 size_t workspace_bytes, void* stream);


/* ------------------------------------------------ int8 tensor engine (tcgen05) */

/* Raw int32 accumulators C[m, n] = A[m, k] . W[n, k]^T (int8, K-major rows;
 * lda / ldw / ldc in elements).  The tensor-engine contract of the reference:
 * torch._int_mm in fixed_mlp._integer_matmul (fixed_mlp.py:55-62) and the
 * int8 MAC tile hls/tensor_engine/int8_mac_tile.cpp:7-41.  A and W must be
 * 16-byte aligned with lda, ldw multiples of 16. */
uint32_t dh_gemm_i8_s32(const int8_t* a, uint64_t lda, const int8_t* w, uint64_t ldw, int32_t* c,
                        uint64_t ldc, uint32_t m, uint32_t n, uint32_t k, void* stream);

/* Integer requantisation on the tensor engine, the RTL arithmetic of
 * fixed_mlp.hardware_requantized_linear (fixed_mlp.py:139-224): C = A . W^T
 * (int8, K-major, k a multiple of 16) and per output
 *   mode 0: mult = rint(double(fp32(a_scale[r] * w_scale[c])) * 2^(right_shift + frac_bits))
 *   mode 1: mult = (token_factor[r] * output_factor[c] + 2^(factor_shift-1)) >> factor_shift
 *           (the factorised multipliers of factorize_up_requant_scales, fixed_mlp.py:327-392)
 *   p = C * mult (int64),  q = sign(p) * ((|p| + 2^(right_shift-1)) >> right_shift)
 *   out = clamp(q + bias_q[c], -2^(output_width-1), 2^(output_width-1) - 1)   (int32 [m, n])
 * a_scale_stride 1: one scale per row (token granularity); 0: a_scale[0] for
 * every row (tensor granularity).  stats (may be NULL; int64[4], initialised by
 * the caller to {INT64_MAX, INT64_MIN, 0, 0}) receives the accumulator minimum
 * and maximum, the number of saturated outputs and the largest multiplier; the
 * caller checks the multiplier width (the reference rejects wider ones). */
uint32_t dh_gemm_i8_requant(const int8_t* a, const int8_t* w, uint32_t m, uint32_t n, uint32_t k,
                            uint32_t mode, const float* a_scale, uint32_t a_scale_stride,
                            const float* w_scale, const int32_t* token_factor,
                            const int32_t* output_factor, uint32_t factor_shift, const int32_t* bias_q,
                            uint32_t right_shift, uint32_t frac_bits, uint32_t output_width,
                            int32_t* out, int64_t* stats, void* stream);

/* RTL Q5.10 GELU lookup (fixed_mlp.hardware_gelu_q10, fixed_mlp.py:227-247):
 * out = 0 for in <= -8192, in for in >= 8192, else lut[(in + 8192) >> 4];
 * lut holds the 1024 table entries. */
uint32_t dh_gelu_q10(const int32_t* in, int32_t* out, uint64_t count, const int32_t* lut, void* stream);

/* ------------------------------------------ RTL fixed-point block stages */
/* Bit-exact integer stages of the RTL DDiT contracts.  Float inputs are
 * converted with round-half-even (torch.round); all other arithmetic is
 * integer, int64 where the reference uses int64 tensors. */

/* fixed_norm.fixed_layer_norm_q12 (fixed_norm.py:13-104): per row of
 * `cols` fp32 values, q = clamp(round(x * 2^in_frac), +-2^23); mean and
 * mean-square with round-half-up integer division; variance clamped at 0;
 * root = isqrt((variance + epsilon_q) << 2*sqrt_extra); inverse =
 * (2^(inv_frac + in_frac + sqrt_extra) + root/2) / root; out =
 * clamp(sym_round_shift((q - mean) * inverse, inv_frac + in_frac - out_frac),
 * +-2^17) as int32 [rows, cols].  row_stats (may be NULL): int64 [rows][5] =
 * mean, variance, inverse, radicand << 2*sqrt_extra, saturated inputs. */
uint32_t dh_fixed_layer_norm_q12(const float* in, uint32_t rows, uint32_t cols, uint32_t input_fraction_bits,
                                 uint32_t output_fraction_bits, uint32_t inverse_fraction_bits,
                                 uint32_t sqrt_extra_fraction_bits, int64_t epsilon_q, int32_t* out,
                                 int64_t* row_stats, void* stream);

/* fixed_attention.fixed_rotary_q12 (fixed_attention.py:24-113): qkv fp32
 * [tokens, 3, heads, 64] -> qkv_q12 (all three, clamped Q5.12) and the
 * rotate-half Q5.12 query / key [tokens, heads, 64] with Q1.15 cosine / sine
 * [tokens, 32].  stats (may be NULL; int64[6], initialised by the caller to
 * 0, 0, INT64_MAX, INT64_MIN, INT64_MAX, INT64_MIN): saturated q/k inputs,
 * saturated v inputs, query min / max, key min / max. */
uint32_t dh_fixed_rotary_q12(const float* qkv, const float* cosine, const float* sine, uint32_t tokens,
                             uint32_t heads, int32_t* qkv_q12, int32_t* query_q12, int32_t* key_q12,
                             int64_t* stats, void* stream);

/* fixed_attention.fixed_attention_q12 (fixed_attention.py:174-298) after the
 * rotary stage: scores = clamp(sym_round_shift(q . k, 17), +-2^17) (Q7.10),
 * delta = clamp(score - row max, -cutoff_q10, 0), exponential =
 * lut[min((-delta + 2^(9 - step_bits)) >> (10 - step_bits), lut_entries - 1)],
 * reciprocal = (2^30 + sum/2) / sum, p = min((e * reciprocal + 2^13) >> 14,
 * 65535), out = clamp(sym_round_shift(sum_s p * v, 16), +-2^17) as int32
 * [tokens, heads * 64].  tokens <= 2048.  scores_q10 / probabilities_q16
 * (may be NULL) receive [heads, tokens, tokens].  stats (may be NULL;
 * int64[5], initialised to 0, INT64_MAX, INT64_MIN, 0, 0): saturated scores,
 * score min / max, minimum delta, maximum |row sum of p - 65536|. */
uint32_t dh_fixed_attention_q12(const int32_t* query_q12, const int32_t* key_q12, const int32_t* qkv_q12,
                                uint32_t tokens, uint32_t heads, uint32_t exponential_step_bits,
                                int64_t cutoff_q10, const int32_t* exponential_lut_q16, uint32_t lut_entries,
                                int32_t* out_q12, int32_t* scores_q10, int32_t* probabilities_q16,
                                int64_t* stats, void* stream);

/* The fixed-point projections (fixed_attention.py:301-494):
 * acc = activation[r] . weight[c] (int64), out = clamp(sym_round_shift(acc *
 * multiplier[c], shift) + bias_q[c], output_min, output_max) as int32
 * [rows, n]; activation int32 [rows, k], weight int16 [n, k] (int8 or int16
 * values), bias_q may be NULL.  accumulators (may be NULL) receive the int64
 * accumulators.  stats (may be NULL; int64[4], initialised to INT64_MAX,
 * INT64_MIN, 0, 0): accumulator min / max, saturated outputs, max |acc|. */
uint32_t dh_fixed_wide_linear(const int32_t* activation, const int16_t* weight, const int64_t* multiplier,
                              const int32_t* bias_q, uint32_t rows, uint32_t n, uint32_t k, uint32_t shift,
                              int64_t output_min, int64_t output_max, int32_t* out, int64_t* accumulators,
                              int64_t* stats, void* stream);

/* The packed INT8 attention candidates of attention_int8.py (:20-315):
 * dynamic_qk_fixed_pv_attention_q12 and _evaluate_with_fixed_maxima after the
 * rotary stage.  Q / K [tokens, heads, 64] (rotated Q5.12) are requantised
 * per qk_mode -- 0 not at all, 1 one calibrated multiplier per head, 2 one
 * maximum per token vector with multiplier rint(qk_levels *
 * 2^qk_fraction_bits / max) (maxima written to query_maxima / key_maxima
 * [tokens, heads]) -- as clamp(sym_round_shift(x * multiplier,
 * qk_fraction_bits), +-qk_levels).  With qk_scores (needs qk_mode != 0),
 * scores = clamp(sym_round_shift(dot * m, 28), +-2^17) with m the per-head
 * calibrated multiplier or rint(q_max * k_max * 2^28 / (qk_levels^2 *
 * 2^17)); else the fixed18 scores of dh_fixed_attention_q12.  Then its LUT
 * softmax.  V is requantised to pv_value_levels (per-head multiplier, 24
 * fraction bits) when that is non-zero.  With pv_probability_levels != 0
 * (needs pv_value_levels), p is requantised to clamp((p * levels + 2^15) >>
 * 16, 0, levels) (the residual levels - sum added at the first largest p
 * when pv_sum_correction) and out = clamp(sym_round_shift(sum p * v *
 * output multiplier, 24), +-2^17); else out = clamp(sym_round_shift(sum p *
 * v_q12, 16), +-2^17).  head_params: int64 [heads][8] = query, key, value
 * multipliers, calibrated score multiplier, output multiplier, query, key,
 * value calibration maxima.  workspace: int32 [3 * tokens * heads * 64]
 * (may be NULL when qk_mode = 0 and pv_value_levels = 0).  Optional outputs
 * (may be NULL): scores_q10, probabilities_q16, probabilities_quantized
 * [heads, tokens, tokens]; head_stats int64 [heads][4] (zeroed by the
 * caller) = query, key and value inputs above their calibration maxima and
 * requantised probabilities of 0 (before the sum correction).
 * tokens <= 2048. */
uint32_t dh_packed_int8_attention_q12(const int32_t* query_q12, const int32_t* key_q12, const int32_t* qkv_q12,
                                      uint32_t tokens, uint32_t heads, uint32_t qk_mode, uint32_t qk_scores,
                                      uint32_t qk_levels, uint32_t qk_fraction_bits, uint32_t pv_probability_levels,
                                      uint32_t pv_sum_correction, uint32_t pv_value_levels,
                                      const int64_t* head_params, uint32_t exponential_step_bits, int64_t cutoff_q10,
                                      const int32_t* exponential_lut_q16, uint32_t lut_entries, int32_t* workspace,
                                      int32_t* out_q12, int32_t* scores_q10, int32_t* probabilities_q16,
                                      int32_t* probabilities_quantized, int32_t* query_maxima,
                                      int32_t* key_maxima, int64_t* head_stats, void* stream);

/* ------------------------------------------------------- DDiT forward path */
/* W8A8 convention (fixed_mlp.quantized_linear, fixed_mlp.py:65-136, with static
 * SmoothQuant scales s per input channel): an activation row a is quantised as
 * a' = a / s (passed here as inv_smooth = 1/s), a_scale = max|a'| / 127
 * (1 if 0), q = clamp(round(a' / a_scale), -127, 127); the linear output is
 * acc * (a_scale * w_scale) + bias with w_scale per output channel.  d = 768,
 * 12 heads x 64, MLP 3072.  `run_flag` / `run_rows` (device words, may be
 * NULL) limit a launch to its first *run_rows rows (the attention: to the
 * sequences those rows cover), so a captured graph skips a forward with 0,
 * or runs it over the sequences that need one, packed first. */

/* x[r, :] = embedding[tokens[r], :]  (fp32 rows of 768; mlx_mdlm.py:262-268). */
uint32_t dh_embed_gather(const int32_t* tokens, const float* embedding, float* x, uint32_t rows,
                         uint32_t vocabulary_size, const uint32_t* run_flag, void* stream);

/* dh_embed_gather over a packed list of sequences: row r of x is position
 * r % positions of sequence seq_list[r / positions] of tokens [*, positions]
 * (the forward of only the sequences that need one; dh_loop_plan_seqs). */
uint32_t dh_embed_gather_seqs(const int32_t* tokens, const uint32_t* seq_list, uint32_t positions,
                              const float* embedding, float* x, uint32_t rows, uint32_t vocabulary_size,
                              const uint32_t* run_rows, void* stream);

/* LayerNorm (no affine, eps 1e-5) -> SmoothQuant division by smooth[768]
 * -> per-token int8 (K3): a = LN(x) / s, scale = amax(|a|) / 127 (1 for a
 * zero row), q = round_half_even(a / scale) clamped to +-127, each quotient
 * the IEEE-rounded fp32 quotient as in fixed_mlp._quantize_symmetric
 * (fixed_mlp.py:11-35) and quantized_linear (:82-90).  inv_smooth (may be
 * NULL) holds the fp32 reciprocals 1/s rounded to nearest: with them the
 * division by s costs three FMAs per element instead of a full division and
 * gives the same quotients (other values than the rounded reciprocals give
 * quotients within an ulp).  The adaLN affine is folded into the following
 * linear (model_specialization.py:10-29).  Optional gather: output row i
 * reads input row rows_index[i] for i < *rows_count. */
uint32_t dh_ln_smooth_quant(const float* x, const float* smooth, const float* inv_smooth, int8_t* out, float* scale,
                            uint32_t rows, const uint32_t* rows_index, const uint32_t* rows_count,
                            const uint32_t* run_flag, void* stream);

/* dh_ln_smooth_quant of packed rows (the forward over seq_list, see
 * dh_embed_gather_seqs), each output row written back to its sequence's own
 * row seq_list[r / positions] * positions + r % positions of out / scale:
 * the head's int8 input of every sequence stays available between the
 * forwards of that sequence. */
uint32_t dh_ln_smooth_quant_scatter(const float* x, const float* smooth, const float* inv_smooth, int8_t* out,
                                    float* scale, uint32_t rows, const uint32_t* seq_list, uint32_t positions,
                                    const uint32_t* run_rows, void* stream);

/* dst row i = src row rows_index[i] (768 int8) and dst_scale[i] =
 * src_scale[rows_index[i]] for i < min(rows, *rows_count). */
uint32_t dh_gather_rows_i8(const int8_t* src, const float* src_scale, const uint32_t* rows_index,
                           const uint32_t* rows_count, uint32_t rows, int8_t* dst, float* dst_scale, void* stream);

/* dst row i = src row rows_index[i] for i < min(rows, *rows_count): rows of
 * row_bytes bytes (a multiple of 16; both buffers 16-byte aligned).  The
 * revealed rows' residual stream and attention output, gathered for the
 * last block, which the loop computes for those rows only. */
uint32_t dh_gather_rows(const void* src, uint32_t row_bytes, const uint32_t* rows_index,
                        const uint32_t* rows_count, uint32_t rows, void* dst, void* stream);

/* bf16 rows (cols = 768 or 3072) -> per-token int8 (K3'), the quantiser of
 * dh_ln_smooth_quant on fp32(in) / smooth (inv_smooth as there).  smooth may
 * be NULL when the producer already applied the SmoothQuant scale (see
 * v_scale / out_scale below). */
uint32_t dh_quant_rows_bf16(const void* in, const float* smooth, const float* inv_smooth, int8_t* out, float* scale,
                            uint32_t rows, uint32_t cols, const uint32_t* run_flag, void* stream);

/* QKV projection (K4): [m, 768] x [2304, 768]^T, dequant, rotate-half rotary
 * on q and k at position (row % seq_len) + pos_offset (mlx_mdlm.py:298-329),
 * written as bf16 Q [B, 12, seq_len, 64] and K [B, 12, kv_stride, 64] and f16
 * V^T [B, 12, 64, kv_stride] at key offset kv_offset (a multiple of 32) --
 * the layout of a cached
 * prefix followed by the active rows (prefix_drift.py:155-238).
 * rope_cos / rope_sin: [positions, 32] fp32.  v_scale (768, may be NULL)
 * multiplies V per channel: with the SmoothQuant 1/s of the attention-out
 * linear, softmax(QK^T)(V diag(1/s)) = (softmax(QK^T) V) diag(1/s) arrives
 * pre-smoothed. */
uint32_t dh_gemm_qkv_rope(const int8_t* a, const float* a_scale, const int8_t* w,
                          const float* w_scale, const float* bias, const float* rope_cos,
                          const float* rope_sin, const float* v_scale, uint32_t m, uint32_t seq_len, uint32_t pos_offset,
                          uint32_t kv_stride, uint32_t kv_offset, void* q, void* k, void* vt,
                          const uint32_t* run_rows, void* stream);

/* x[m, n] += dequant(A . W^T) (+ bias): attention-out (K6) and MLP-down (K8),
 * with the adaLN gates folded into W and bias (mlx_mdlm.py:442-453). */
uint32_t dh_gemm_residual(const int8_t* a, const float* a_scale, const int8_t* w,
                          const float* w_scale, const float* bias, float* x, uint32_t m, uint32_t n,
                          uint32_t k, const uint32_t* run_rows, void* stream);

/* out[m, n] = bf16(gelu_tanh(dequant(A . W^T) + bias) * out_scale[n]): MLP-up
 * (K7); out_scale (may be NULL) is the SmoothQuant 1/s of MLP-down.
 * row_amax (device uint32 [m], may be NULL; must hold 0 on entry): the bits
 * of each row's max |out| (non-negative fp32, so atomicMax on the bits orders
 * them) for dh_quant_rows_bf16_amax.  n is a multiple of 256 and at most
 * 3584 (the column parameters stay in shared memory);
 * DH_ERR_UNSUPPORTED_SHAPE otherwise. */
uint32_t dh_gemm_gelu(const int8_t* a, const float* a_scale, const int8_t* w,
                      const float* w_scale, const float* bias, const float* out_scale, void* out,
                      uint32_t* row_amax, uint32_t m, uint32_t n,
                      uint32_t k, const uint32_t* run_rows, void* stream);

/* The per-token quantiser of dh_quant_rows_bf16 (no smoothing) for bf16 rows
 * whose max |x| the producer already left in row_amax (dh_gemm_gelu): one
 * streaming pass instead of two, the same bytes and scales; row_amax[r] is
 * reset to 0 afterwards.  cols a multiple of 256. */
uint32_t dh_quant_rows_bf16_amax(const void* in, uint32_t* row_amax, int8_t* out, float* scale, uint32_t rows,
                                 uint32_t cols, const uint32_t* run_flag, void* stream);

/* Bidirectional attention softmax(Q K^T / 8) V (K5) over the first kv_len
 * keys of K / V^T buffers of kv_stride rows per (sequence, head); Q, K bf16,
 * V^T f16, fp32 scores and row sums, P in f16, bf16 out [sequences * q_len, 768].  q_len, kv_len multiples
 * of 32, kv_stride a multiple of 8.  Keys are read in tiles of 64: when
 * kv_len is not a multiple of 64, the V^T columns from kv_len up to the next
 * multiple of 64 that lie inside kv_stride must hold finite values (zero-fill
 * the buffers once); those keys are masked. */
uint32_t dh_attention(const void* q, const void* k, const void* vt, void* out, uint32_t sequences,
                      uint32_t q_len, uint32_t kv_len, uint32_t kv_stride, const uint32_t* run_flag,
                      void* stream);

/* ---------------------------- final layer with per-sequence conditioning */

/* adaLN modulation of the final layer (mlx_mdlm._FinalLayer.prepare,
 * mlx_mdlm.py:466-471): out[b, n] = bias[n] + sum_c cond[b, c] weight[n, c]
 * (fp32, c summed in order); with outputs = 2 d the first d are the shift,
 * the next d the scale.  bias may be NULL. */
uint32_t dh_adaln_modulation(const float* cond, const float* weight, const float* bias, float* out,
                             uint32_t sequences, uint32_t condition_size, uint32_t outputs, void* stream);

/* The head's input when the conditioning varies per sequence
 * (mlx_mdlm._FinalLayer.hidden, mlx_mdlm.py:487-493, then the per-token
 * int8 of fixed_mlp._quantize_symmetric, fixed_mlp.py:11-35): for output row
 * i < min(rows, *rows_count) the hidden row r = rows_index[i] (bf16 [*, 768];
 * identity when rows_index is NULL) of sequence b = r / rows_per_sequence is
 * LayerNorm-ed (eps 1e-5, times ln_weight, NULL = ones), modulated
 * h = n (1 + scale_b) + shift_b with modulation[b] = [shift | scale] (fp32
 * [sequences, 1536], dh_adaln_modulation), and quantised per token: out[i]
 * int8 [768] and scale[i] = amax / 127. */
uint32_t dh_ln_modulate_quant_bf16(const void* hidden, const float* ln_weight, const float* modulation,
                                   uint32_t rows_per_sequence, const uint32_t* rows_index,
                                   const uint32_t* rows_count, uint32_t rows, int8_t* out, float* scale,
                                   void* stream);

/* ------------------------------------------------ fused int8 head (K9) */

/* Head + noisy argmax over `rows` int8 hidden rows (ld_hidden bytes apart)
 * and the int8 [vocab, hidden_size] weight (ld_weights bytes per row), on
 * tcgen05; logits never leave the chip.  Per row, the best (score, lowest id)
 * is merged into packed[row] (zeroed by this call) and, if given, written to
 * out_ids / out_scores.  mode 0: HLS requant score, requant_q20(acc,
 * mult_q20[v]) + bias_q10[v] + noise (output_head.cpp:126-146); mode 1: the
 * reference W8A8 logit float(double(acc) * double(a_scale[r]*w_scale[v]) +
 * double(bias[v])) (fixed_mlp.py:98-106), Q10-rounded (rng.py:262), + noise;
 * mode 2: argmax of that fp32 logit (greedy pass, mdlm.py:1190).  noise is
 * the given [rows, vocab] array or the factorized Gumbel of
 * philox((v/4, row_position[r], row_eval[r] or const_eval, stream_id),
 * (key_lo, row_key_hi[r]))[v%4].  rows_count (device, may be NULL) limits the
 * rows processed, for data-dependent row sets.  Mask token skipped.
 * Vocab-sharded head: `weights` / `w_scale` / `bias` hold the rows of global
 * tokens [vocab_offset, vocab_offset + vocabulary_size) (vocab_offset a
 * multiple of 4); ids, noise counters and the mask test use global ids (the
 * mask id may lie outside the shard), so a
 * MAX reduction of the packed words over shards gives the unsharded result
 * (the tie rule of ordered_noisy_argmax_reducer.sv:106-133 included).
 * Status: head family codes, then DH_ERR_*. */
uint32_t dh_head_argmax_i8(const int8_t* hidden, uint64_t ld_hidden, const int8_t* weights,
                           uint64_t ld_weights, uint32_t rows, const uint32_t* rows_count,
                           uint32_t hidden_size, uint32_t vocabulary_size, uint32_t vocab_offset,
                           uint32_t mask_token_id, uint32_t mode, const float* a_scale, const float* w_scale,
                           const float* bias, const int32_t* mult_q20, const int32_t* bias_q10,
                           const int32_t* noise, const uint32_t* row_position,
                           const uint32_t* row_key_hi, const uint32_t* row_eval,
                           uint32_t const_eval, uint32_t key_lo, uint32_t stream_id,
                           uint64_t* packed, int32_t* out_ids, int32_t* out_scores, void* stream);

/* The noise half of dh_head_argmax_i8 alone: per row, the (score, lowest id)
 * race of the Philox / Gumbel Q10 noise with every logit zero (the same
 * counters, key, table and tie rule; mask token skipped), merged into
 * packed[row] (zero on entry) and, if given, out_ids.  Equals
 * dh_noisy_argmax_f32 of all-zero logits.  With no GEMM or logit to compute,
 * its time over the head's rows and vocabulary is the cost of the noise with
 * the integer pipes to itself: the floor of the fused head on the SMs'
 * integer units.  Status: RNG family codes, then DH_ERR_*. */
uint32_t dh_noise_argmax(uint32_t rows, uint32_t vocabulary_size, uint32_t mask_token_id,
                         const uint32_t* row_position, const uint32_t* row_key_hi, const uint32_t* row_eval,
                         uint32_t const_eval, uint32_t const_key_hi, uint32_t key_lo, uint32_t stream_id,
                         uint64_t* packed, int32_t* out_ids, void* stream);

/* Mirror of output_head_int8_kernel (output_head.cpp:23-157): same arguments,
 * limits and status codes (1 <= positions <= 64, 1 <= hidden <= 768,
 * 1 <= vocab <= 65535, mask < vocab); `noise` is the [positions, vocab] race
 * noise or NULL to generate it in place exactly as philox_gumbel_stream_kernel
 * orders it (counter (v/4, position, evaluation_id, stream_id), key
 * (seed_low, seed_high)).  hidden_size must be a multiple of 16 (zero-pad).
 * workspace: position_count uint64 words. */
uint32_t dh_output_head_int8(const int8_t* hidden, const int8_t* weights,
                             const int32_t* requant_multiplier_q20, const int32_t* bias,
                             const int32_t* noise, uint16_t* candidate_ids,
                             uint32_t position_count, uint32_t hidden_size,
                             uint32_t vocabulary_size, uint32_t mask_token_id,
                             uint32_t evaluation_id, uint32_t stream_id, uint32_t seed_low,
                             uint32_t seed_high, uint64_t* workspace, void* stream);

/* ------------------------------------ model loop (selected-row head) state */
/*
 * Device state of the candidate-cache loop around the model, B sequences x L
 * positions: tokens int32 [B*L]; active uint64 [B*W] (W = ceil(L/64));
 * need_eval / eval_id uint32 [B]; counters int32 [3*steps] (per transition:
 * batch active count, changed count, 1 if a forward ran); fwd_rows and
 * sel_count are single device words; sel_rows / sel_pos / sel_key / sel_eval
 * uint32 [B*L] hold the rows revealed at the current transition.
 * Per transition k: dh_loop_plan -> (forward if *fwd_rows) -> dh_loop_select ->
 * dh_ln_smooth_quant (gathering sel_rows) -> dh_head_argmax_i8 (mode 1, rows
 * limited by sel_count) -> dh_loop_commit.  final_pass = 1 runs the greedy
 * pass of mdlm.py:1177-1200 over every still-masked position.
 * Randomness is keyed by the global sequence (seq_offset + b) and the canvas
 * position (position_offset + p): a suffix-only loop over positions
 * [P, P + S) draws the same words as a loop over the whole [0, P + S) canvas.
 */
uint32_t dh_loop_init(const int32_t* input_ids, uint32_t sequences, uint32_t positions,
                      uint32_t mask_token_id, uint32_t steps, int32_t* tokens, uint64_t* active,
                      uint32_t* need_eval, uint32_t* eval_id, int32_t* counters, void* stream);
uint32_t dh_loop_plan(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t steps,
                      uint32_t final_pass, const uint64_t* active, uint32_t* need_eval,
                      uint32_t* eval_id, uint32_t* fwd_rows, uint32_t* sel_count,
                      int32_t* counters, void* stream);
/* dh_loop_plan that also lists the sequences that refill at this transition
 * (seq_list [sequences], ascending) and sets *fwd_rows = their count *
 * positions: the ddpm_cache skip per sequence (mdlm.py:1134-1174 invalidates
 * the cache of a canvas that changed), so the forward covers only those. */
uint32_t dh_loop_plan_seqs(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t steps,
                           uint32_t final_pass, const uint64_t* active, uint32_t* need_eval,
                           uint32_t* eval_id, uint32_t* fwd_rows, uint32_t* sel_count,
                           int32_t* counters, uint32_t* seq_list, void* stream);
uint32_t dh_loop_select(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t seed,
                        uint32_t seq_offset, uint32_t position_offset, uint64_t threshold_q32, uint32_t final_pass, const uint64_t* active,
                        const uint32_t* eval_id, uint32_t* sel_rows, uint32_t* sel_pos,
                        uint32_t* sel_key, uint32_t* sel_eval, uint32_t* sel_count, void* stream);
uint32_t dh_loop_commit(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t steps,
                        uint32_t final_pass, const uint64_t* packed, const uint32_t* sel_rows,
                        const uint32_t* sel_count, int32_t* tokens, uint64_t* active,
                        uint32_t* need_eval, int32_t* counters, void* stream);

/* ------------------------------------------ composite entry points (C ABI) */
/*
 * The whole forward and the whole generation enqueued by the library on one
 * stream, for hosts that do not orchestrate the per-kernel entry points
 * above themselves.  Weights are device pointers gathered in the structs
 * below (the host array `block_linears` holds 4 linears per block: qkv, out,
 * up, down).  Workspaces are caller-owned device buffers, 256-byte aligned,
 * of the size the matching *_workspace_size query returns; nothing is
 * allocated.  Arguments are checked before anything is enqueued.
 */
typedef struct dh_linear_weights {
    const int8_t* weight;     /* [out_features, in_features] int8, per-output-channel quantised */
    const float* w_scale;     /* [out_features] */
    const float* bias;        /* [out_features] fp32; required for qkv and up, may be NULL for out and down */
    const float* smooth;      /* [in_features] SmoothQuant divisor s of this linear's input */
    const float* inv_smooth;  /* [in_features] 1 / s (folded into the producer of out's / down's input) */
} dh_linear_weights;

typedef struct dh_mdlm_weights {
    uint32_t blocks;                          /* DDiT blocks (d = 768, 12 x 64 heads, MLP 3072) */
    uint32_t vocabulary_size;                 /* embedding rows = global vocabulary, mask id included */
    uint32_t mask_token_id;
    uint32_t max_positions;                   /* rows of rope_cos / rope_sin */
    const float* embedding;                   /* [vocabulary_size, 768] fp32 */
    const float* rope_cos;                    /* [max_positions, 32] fp32 */
    const float* rope_sin;
    const dh_linear_weights* block_linears;   /* HOST array [blocks * 4] */
    dh_linear_weights head;                   /* head rows [head_vocab_offset, + head_rows) of [V, 768] */
    uint32_t head_rows;                       /* the whole vocabulary, or this rank's shard */
    uint32_t head_vocab_offset;               /* global id of head row 0, a multiple of 4 */
} dh_mdlm_weights;

/* The folded W8A8 DDiT forward (hardware_package.folded_mdlm_forward,
 * hardware_package.py:195-289; per block the kernels dh_ln_smooth_quant,
 * dh_gemm_qkv_rope, dh_attention, dh_quant_rows_bf16, dh_gemm_residual,
 * dh_ln_smooth_quant, dh_gemm_gelu, dh_quant_rows_bf16, dh_gemm_residual)
 * of `sequences` x `positions` token ids (device int32, positions a multiple
 * of 32, full bidirectional attention, rotary positions 0..positions-1).
 * x (device fp32 [sequences * positions, 768]) receives the residual stream
 * after the last block, before the final LayerNorm.  run_rows (device word,
 * may be NULL): the forward does nothing when it holds 0. */
size_t dh_ddit_forward_workspace_size(uint32_t sequences, uint32_t positions);
uint32_t dh_ddit_forward(const dh_mdlm_weights* weights, const int32_t* tokens, uint32_t sequences,
                         uint32_t positions, float* x, void* workspace, size_t workspace_bytes,
                         const uint32_t* run_rows, void* stream);

/* The candidate-cache generation of mdlm._run_ddpm_candidate_cache_sampler
 * (mdlm.py:1104-1218) over the model: input_ids (device int32 [sequences *
 * positions], masked positions = mask_token_id) -> tokens (device int32, same
 * shape; the loop's canvas), `steps` transitions and the final greedy pass,
 * with the reveal threshold of transition k thresholds_q32[k] (HOST array,
 * min(2^32, floor(p_k 2^32)) for the schedule's reveal probability p_k,
 * mdlm.py:1116-1117, 1151-1153) and the noise / reveal words keyed by
 * (seed, seq_offset + b) as in dh_loop_select and dh_head_argmax_i8.
 * counters (device int32 [3 * steps]): per transition the active count, the
 * changed count and 1 if the model ran (the reference's metadata).
 * nccl_comm: NULL, or the ncclComm_t of the ranks that hold the vocabulary
 * shards of the head (weights->head_rows / head_vocab_offset); after every
 * head launch the packed per-row results are merged by
 * dh_vocab_shard_reduce over it, so every rank commits the unsharded argmax.
 * compact: 0 -> a transition runs the forward over the whole batch when any
 * sequence refills; 1 -> only over the sequences that refill, packed
 * (dh_loop_plan_seqs), with every refilled row's head input kept per
 * sequence -- the same tokens, fewer rows when canvases are small (a
 * sequence with L/steps expected reveals per transition skips one with
 * probability about exp(-L/steps)), one extra LayerNorm pass over the
 * refilled rows otherwise.  The whole generation is enqueued without host
 * synchronisation (it can be captured in a CUDA graph).  Status:
 * DH_CAND_INVALID_THRESHOLD for a threshold above 2^32, else DH_ERR_*. */
size_t dh_sample_loop_workspace_size(uint32_t sequences, uint32_t positions);
uint32_t dh_sample_loop(const dh_mdlm_weights* weights, const int32_t* input_ids, int32_t* tokens,
                        uint32_t sequences, uint32_t positions, uint32_t steps, const uint64_t* thresholds_q32,
                        uint32_t seed, uint32_t seq_offset, int32_t* counters, void* nccl_comm, uint32_t compact,
                        void* workspace, size_t workspace_bytes, void* stream);

/* Merge of the vocab-sharded head: packed (device uint64 [count], as written
 * by dh_head_argmax_i8: (score ^ 2^31) << 32 | ~id) is MAX-all-reduced in
 * place over nccl_comm (an ncclComm_t; the NCCL library that created it must
 * be loaded in the process, its ncclAllReduce is used) on `stream`.  The
 * unsigned order of the packed words is the order of (score, lower id), the
 * tie rule of ordered_noisy_argmax_reducer.sv:106-133.  DH_ERR_NCCL when
 * NCCL is not loaded or the call fails. */
uint32_t dh_vocab_shard_reduce(void* nccl_comm, uint64_t* packed, uint64_t count, void* stream);

/* ------------------------------------------------------------- diagnostics */

/* Reads (and optionally clears) the device error word.  Non-zero means a
 * bounded wait inside a kernel expired (1..4: pipeline barrier that timed
 * out); the kernel abandoned its work and its outputs are undefined.
 * Synchronous. */
uint32_t dh_device_error(uint32_t* out, uint32_t clear);

/* Self-check of the bounded waits (failure detection without a GPU fault):
 * one thread waits on an mbarrier whose single arrival is made only when
 * `arrive` != 0.  Without it the wait gives up after spin_limit polls
 * (1 <= spin_limit <= 65536), sets the device error word to 1 (the code of
 * an expired pipeline wait) and the kernel returns; *completed (device word)
 * is 1 if the wait completed, else 0.  No counterpart in the reference, whose
 * HLS kernels report status codes but have no device waits. */
uint32_t dh_wait_selftest(uint32_t spin_limit, uint32_t arrive, uint32_t* completed, void* stream);

/* The same check for the suspending waits (the attention kernel's): the
 * waiting thread sleeps on the mbarrier and gives up after limit_ns
 * nanoseconds of wall time (1 <= limit_ns <= 2e9, the kernels' own bound),
 * with the same error word and *completed as dh_wait_selftest. */
uint32_t dh_wait_suspend_selftest(uint64_t limit_ns, uint32_t arrive, uint32_t* completed, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* DH_B200_H */
