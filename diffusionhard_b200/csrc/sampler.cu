// sampler.cu -- Philox/Gumbel streams, Gumbel-max over fp32 logits (K1),
// candidate reveal (K2) and the device-resident candidate-cache transition.
//
// Reference semantics:
//   Philox word/score streams     hls/rng/philox_rng.cpp:95-205
//   noisy argmax (Q10 race)       src/diffusion_accel/rng.py:262-263,
//                                 hls/output_head/output_head.cpp:138-151
//   candidate reveal              hls/candidate_sampler/candidate_sampler.cpp:5-79
//   candidate-cache transition    src/diffusion_accel/mdlm.py:1104-1218
//
// All of these are HBM- or latency-bound integer kernels: coalesced loads,
// grids sized by rows x vocab chunks, no tensor cores.
#include <cuda.h>

#include "dh_common.cuh"
#include "dh_philox.cuh"

#include <algorithm>
#include <mutex>

namespace dh {
namespace {

constexpr uint32_t kArgmaxThreads = 256;
constexpr uint32_t kArgmaxGroupsPerThread = 4;
constexpr uint32_t kArgmaxChunk = kArgmaxThreads * kArgmaxGroupsPerThread * 4;  // 4096 tokens

DH_DEVINL int32_t logit_q10(float logit) {
    const float scaled = __fmul_rn(logit, 1024.0f);
    if (!(scaled == scaled)) return -(1 << 30);
    if (scaled > 1073741824.0f) return 1 << 30;
    if (scaled < -1073741824.0f) return -(1 << 30);
    return __float2int_rn(scaled);
}

__global__ void philox_batch_kernel(const uint32_t* __restrict__ ctr,
                                    const uint32_t* __restrict__ key, uint32_t* __restrict__ out,
                                    uint32_t count) {
    const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= count) return;
    Philox4 r = philox4x32_10(ctr[4 * i], ctr[4 * i + 1], ctr[4 * i + 2], ctr[4 * i + 3],
                              key[2 * i], key[2 * i + 1]);
    out[4 * i] = r.x;
    out[4 * i + 1] = r.y;
    out[4 * i + 2] = r.z;
    out[4 * i + 3] = r.w;
}

__global__ void gumbel_batch_kernel(const uint32_t* __restrict__ words, int32_t* __restrict__ out,
                                    uint32_t count) {
    __shared__ __align__(16) int16_t table[32 * 256];
    load_gumbel_table(table);
    __syncthreads();
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < count;
         i += gridDim.x * blockDim.x)
        out[i] = gumbel_q10(words[i], table);
}

// One thread per (position, group of 4 tokens); writes up to 4 entries at the
// reference stream index  P*vbase + p*tile_len + (t - vbase),  vbase = t & ~15.
template <bool kScores>
__global__ void philox_stream_kernel(void* __restrict__ out, uint32_t positions, uint32_t vocab,
                                     uint32_t eval_id, uint32_t stream_id, uint32_t seed_lo,
                                     uint32_t seed_hi) {
    __shared__ __align__(16) int16_t table[32 * 256];
    if (kScores) {
        load_gumbel_table(table);
        __syncthreads();
    }
    const uint32_t groups = (vocab + 3) / 4;
    const uint64_t total = static_cast<uint64_t>(groups) * positions;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint32_t p = static_cast<uint32_t>(i / groups);
        const uint32_t g = static_cast<uint32_t>(i % groups);
        const uint32_t t0 = g * 4;
        Philox4 r = philox4x32_10(g, p, eval_id, stream_id, seed_lo, seed_hi);
        const uint32_t vbase = t0 & ~15u;
        const uint32_t tile_len = min(16u, vocab - vbase);
        const uint64_t base = static_cast<uint64_t>(positions) * vbase +
                              static_cast<uint64_t>(p) * tile_len + (t0 - vbase);
#pragma unroll
        for (uint32_t w = 0; w < 4; ++w) {
            if (t0 + w >= vocab) break;
            const uint32_t word = philox_lane(r, w);
            if (kScores)
                static_cast<int32_t*>(out)[base + w] = gumbel_q10(word, table);
            else
                static_cast<uint32_t*>(out)[base + w] = word;
        }
    }
}

// ---------------------------------------------------------------- K1 argmax

struct ArgmaxRows {
    const float* logits;
    uint64_t row_stride;
    uint32_t rows, vocab, mask_id;
    // Per-row counter metadata.  When an array is NULL the value is derived
    // from the row index: position = r % seq_positions (or r), key_hi =
    // r / seq_positions (or 0), eval = const_eval.
    const uint32_t* row_position;
    const uint32_t* row_key_hi;
    const uint32_t* row_eval;
    uint32_t key_lo, stream_id;
    uint32_t seq_positions;
    uint32_t const_eval;
    // Optional gates: row r is processed only if seq_gate[r / seq_positions]
    // is non-zero and (when `active` is given) its active bit is set.
    const uint32_t* seq_gate;
    const uint64_t* active;
};

DH_DEVINL bool row_enabled(const ArgmaxRows& a, uint32_t r) {
    if (a.seq_gate && a.seq_gate[r / a.seq_positions] == 0u) return false;
    if (a.active && ((a.active[r >> 6] >> (r & 63u)) & 1ull) == 0ull) return false;
    return true;
}

DH_DEVINL uint32_t row_pos_of(const ArgmaxRows& a, uint32_t r) {
    return a.row_position ? a.row_position[r] : (a.seq_positions ? r % a.seq_positions : r);
}
DH_DEVINL uint32_t row_key_of(const ArgmaxRows& a, uint32_t r) {
    return a.row_key_hi ? a.row_key_hi[r] : (a.seq_positions ? r / a.seq_positions : 0u);
}
DH_DEVINL uint32_t row_eval_of(const ArgmaxRows& a, uint32_t r) {
    return a.row_eval ? a.row_eval[r] : a.const_eval;
}

// Grid (chunks, rows): each block reduces 4096 tokens of one row to one packed
// (score, ~id) and stores it in partial[row * chunks + chunk].
template <bool kNoisy>
__global__ void __launch_bounds__(kArgmaxThreads)
argmax_partial_kernel(ArgmaxRows a, uint64_t* __restrict__ partial, uint32_t chunks) {
    __shared__ __align__(16) int16_t table[32 * 256];
    __shared__ uint64_t warp_best[kArgmaxThreads / 32];
    const uint32_t r = blockIdx.y;
    const uint32_t chunk = blockIdx.x;
    if (!row_enabled(a, r)) return;
    if (kNoisy) {
        load_gumbel_table(table);
        __syncthreads();
    }
    const float* row = a.logits + static_cast<uint64_t>(r) * a.row_stride;
    const uint32_t pos = row_pos_of(a, r);
    const uint32_t key_hi = row_key_of(a, r);
    const uint32_t ev = row_eval_of(a, r);
    uint64_t best = 0;
#pragma unroll 1
    for (uint32_t j = 0; j < kArgmaxGroupsPerThread; ++j) {
        const uint32_t t0 = chunk * kArgmaxChunk + (j * kArgmaxThreads + threadIdx.x) * 4;
        if (t0 >= a.vocab) break;
        Philox4 w{0, 0, 0, 0};
        if (kNoisy) w = philox4x32_10(t0 >> 2, pos, ev, a.stream_id, a.key_lo, key_hi);
#pragma unroll
        for (uint32_t i = 0; i < 4; ++i) {
            const uint32_t t = t0 + i;
            if (t >= a.vocab || t == a.mask_id) continue;
            const float l = __ldg(row + t);
            uint64_t packed;
            if (kNoisy)
                packed = pack_score_id(logit_q10(l) + gumbel_q10(philox_lane(w, i), table), t);
            else
                packed = pack_float_id(l, t);
            best = packed > best ? packed : best;
        }
    }
    best = warp_max_u64(best);
    if (lane_id() == 0) warp_best[warp_id()] = best;
    __syncthreads();
    if (threadIdx.x == 0) {
        uint64_t b = warp_best[0];
        for (uint32_t w = 1; w < kArgmaxThreads / 32; ++w) b = warp_best[w] > b ? warp_best[w] : b;
        partial[static_cast<uint64_t>(r) * chunks + chunk] = b;
    }
}

// One warp per row: reduce the chunk partials.  Writes ids / scores, and for
// the sampler the candidate (uint16) or the committed greedy token.
enum FinalizeMode : uint32_t { kFinalizeIds = 0, kFinalizeCandidates = 1, kFinalizeGreedyCommit = 2 };

__global__ void argmax_finalize_kernel(ArgmaxRows a, const uint64_t* __restrict__ partial,
                                       uint32_t chunks, uint32_t mode, bool noisy,
                                       int32_t* __restrict__ out_ids,
                                       int32_t* __restrict__ out_scores,
                                       uint16_t* __restrict__ candidates) {
    const uint32_t r = blockIdx.x * (blockDim.x / 32) + warp_id();
    if (r >= a.rows) return;
    if (!row_enabled(a, r)) return;
    uint64_t best = 0;
    for (uint32_t c = lane_id(); c < chunks; c += 32) {
        const uint64_t v = partial[static_cast<uint64_t>(r) * chunks + c];
        best = v > best ? v : best;
    }
    best = warp_max_u64(best);
    if (lane_id() != 0) return;
    const uint32_t id = best == 0 ? 0u : packed_id(best);
    if (mode == kFinalizeIds) {
        out_ids[r] = static_cast<int32_t>(id);
        if (out_scores) {
            if (noisy) {
                out_scores[r] = packed_score(best);
            } else {
                const uint32_t k = static_cast<uint32_t>(best >> 32);
                const uint32_t bits = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
                out_scores[r] = static_cast<int32_t>(bits);
            }
        }
    } else if (mode == kFinalizeCandidates) {
        candidates[r] = static_cast<uint16_t>(id);
    } else {
        out_ids[r] = static_cast<int32_t>(id);  // tokens
    }
}

// --------------------------------------------------------------- K2 reveal

// Reveal over one sequence per block; a warp owns one 64-bit bitmap word at a
// time (lane l handles positions 64w + l and 64w + 32 + l), so bitmap updates
// need no atomics.  kSampler: int32 tokens, in-kernel reveal words, refill of
// the valid bitmap for sequences whose cache was just refilled.
template <typename Token, bool kSampler>
__global__ void reveal_kernel(Token* __restrict__ tokens, const uint16_t* __restrict__ cands,
                              uint64_t* __restrict__ active, uint64_t* __restrict__ valid,
                              const uint32_t* __restrict__ words, uint64_t threshold,
                              uint32_t positions, uint64_t* __restrict__ results,
                              const uint32_t* __restrict__ refill, uint32_t* __restrict__ eval_id,
                              uint32_t seed, uint32_t step, int32_t* __restrict__ counters) {
    __shared__ uint32_t changed_total;
    const uint32_t s = blockIdx.x;
    const uint32_t nwords = (positions + 63) / 64;
    uint64_t* act = active + static_cast<uint64_t>(s) * nwords;
    uint64_t* val = valid + static_cast<uint64_t>(s) * nwords;
    Token* tok = tokens + static_cast<uint64_t>(s) * positions;
    const uint16_t* cand = cands + static_cast<uint64_t>(s) * positions;
    if (threadIdx.x == 0) changed_total = 0;
    if (kSampler && refill[s]) {
        for (uint32_t w = threadIdx.x; w < nwords; w += blockDim.x) {
            const uint32_t n = min(64u, positions - w * 64);
            val[w] = n == 64 ? ~0ull : ((1ull << n) - 1ull);
        }
        if (threadIdx.x == 0) eval_id[s] = step;
    }
    __syncthreads();
    uint32_t changed = 0;
    for (uint32_t w = warp_id(); w < nwords; w += blockDim.x / 32) {
        const uint64_t a = act[w];
        const uint64_t v = val[w];
        uint32_t take[2];
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
            const uint32_t bit = lane_id() + 32 * h;
            const uint32_t p = w * 64 + bit;
            take[h] = 0;
            if (p < positions && ((a & v) >> bit) & 1ull) {
                uint32_t word;
                if (kSampler) {
                    Philox4 r = philox4x32_10(p >> 2, 0u, step, 1u, seed, s);
                    word = philox_lane(r, p & 3u);
                } else {
                    word = words[static_cast<uint64_t>(s) * positions + p];
                }
                if (static_cast<uint64_t>(word) < threshold) {
                    tok[p] = static_cast<Token>(cand[p]);
                    take[h] = 1;
                }
            }
        }
        const uint32_t lo = __ballot_sync(0xFFFFFFFFu, take[0]);
        const uint32_t hi = __ballot_sync(0xFFFFFFFFu, take[1]);
        const uint64_t mask = (static_cast<uint64_t>(hi) << 32) | lo;
        if (lane_id() == 0 && mask) {
            act[w] = a & ~mask;
            changed += __popcll(mask);
        }
    }
    if (lane_id() == 0 && changed) atomicAdd(&changed_total, changed);
    __syncthreads();
    const uint32_t total = changed_total;
    if (total) {
        for (uint32_t w = threadIdx.x; w < nwords; w += blockDim.x) val[w] = 0ull;
    }
    if (threadIdx.x == 0) {
        if (results) results[s] = total;
        if (kSampler && total) atomicAdd(&counters[3 * step + 1], static_cast<int32_t>(total));
    }
}

// Per sequence (one warp each): active count, refill decision, step counters.
__global__ void sampler_plan_kernel(const uint64_t* __restrict__ active,
                                    const uint64_t* __restrict__ valid, uint32_t sequences,
                                    uint32_t positions, uint32_t step,
                                    uint32_t* __restrict__ refill, int32_t* __restrict__ counters) {
    const uint32_t s = blockIdx.x * (blockDim.x / 32) + warp_id();
    if (s >= sequences) return;
    const uint32_t nwords = (positions + 63) / 64;
    uint32_t count = 0;
    uint32_t any_valid = 0;
    for (uint32_t w = lane_id(); w < nwords; w += 32) {
        count += __popcll(active[static_cast<uint64_t>(s) * nwords + w]);
        any_valid |= valid[static_cast<uint64_t>(s) * nwords + w] != 0ull;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        count += __shfl_xor_sync(0xFFFFFFFFu, count, o);
        any_valid |= __shfl_xor_sync(0xFFFFFFFFu, any_valid, o);
    }
    if (lane_id() == 0) {
        const uint32_t r = (count > 0 && !any_valid) ? 1u : 0u;
        refill[s] = r;
        if (count) atomicAdd(&counters[3 * step], static_cast<int32_t>(count));
        if (r) atomicMax(&counters[3 * step + 2], 1);
    }
}

__global__ void sampler_init_kernel(const int32_t* __restrict__ input_ids, uint32_t sequences,
                                    uint32_t positions, uint32_t mask_id, uint32_t steps,
                                    int32_t* __restrict__ tokens, uint16_t* __restrict__ cands,
                                    uint64_t* __restrict__ active, uint64_t* __restrict__ valid,
                                    uint32_t* __restrict__ eval_id, int32_t* __restrict__ counters) {
    const uint32_t s = blockIdx.x;
    const uint32_t nwords = (positions + 63) / 64;
    for (uint32_t w = warp_id(); w < nwords; w += blockDim.x / 32) {
        uint32_t m[2];
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
            const uint32_t p = w * 64 + lane_id() + 32 * h;
            m[h] = 0;
            if (p < positions) {
                const uint64_t i = static_cast<uint64_t>(s) * positions + p;
                const int32_t t = input_ids[i];
                tokens[i] = t;
                cands[i] = 0;
                m[h] = static_cast<uint32_t>(t) == mask_id;
            }
        }
        const uint32_t lo = __ballot_sync(0xFFFFFFFFu, m[0]);
        const uint32_t hi = __ballot_sync(0xFFFFFFFFu, m[1]);
        if (lane_id() == 0) {
            active[static_cast<uint64_t>(s) * nwords + w] = (static_cast<uint64_t>(hi) << 32) | lo;
            valid[static_cast<uint64_t>(s) * nwords + w] = 0ull;
        }
    }
    if (threadIdx.x == 0) eval_id[s] = 0;
    if (s == 0)
        for (uint32_t i = threadIdx.x; i < 3 * steps; i += blockDim.x) counters[i] = 0;
}

// Clears the active bit of every position (the greedy pass commits them all).
__global__ void clear_bitmap_kernel(uint64_t* __restrict__ bits, uint64_t count) {
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < count;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
        bits[i] = 0ull;
}

uint32_t argmax_chunks(uint32_t vocab) { return (vocab + kArgmaxChunk - 1) / kArgmaxChunk; }

uint32_t launch_argmax(const ArgmaxRows& a, bool noisy, uint32_t mode, int32_t* out_ids,
                       int32_t* out_scores, uint16_t* candidates, void* workspace,
                       cudaStream_t st) {
    const uint32_t chunks = argmax_chunks(a.vocab);
    uint64_t* partial = static_cast<uint64_t*>(workspace);
    dim3 grid(chunks, a.rows);
    if (noisy)
        argmax_partial_kernel<true><<<grid, kArgmaxThreads, 0, st>>>(a, partial, chunks);
    else
        argmax_partial_kernel<false><<<grid, kArgmaxThreads, 0, st>>>(a, partial, chunks);
    DH_LAUNCH_CHECK();
    const uint32_t warps = 8;
    argmax_finalize_kernel<<<(a.rows + warps - 1) / warps, warps * 32, 0, st>>>(
        a, partial, chunks, mode, noisy, out_ids, out_scores, candidates);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

// ------------------------------------------------ no-allocation variant of K1
//
// Scratch of dh_noisy_argmax_f32_noalloc: the per-(row, vocab chunk) partial
// maxima live in this file-scope array instead of a caller workspace.  Every
// GPU that loads the library holds these 512 KiB until the process exits.
// Host code must not use the array's name as a device address: the address is
// resolved once per device with cudaGetSymbolAddress.
constexpr uint32_t kNoAllocScratchWords = 1u << 16;  // 65,536 x 8 bytes = 512 KiB
static __device__ __align__(256) uint64_t g_noalloc_argmax_scratch[kNoAllocScratchWords];

constexpr int kMaxDevices = 64;

// Unique id of the context current on this thread, 0 when there is none or
// the driver does not provide the query.  The driver functions are reached
// through cudaGetDriverEntryPoint, so the library binds no libcuda symbol.
unsigned long long current_context_id() {
    typedef CUresult (*GetCurrentFn)(CUcontext*);
    typedef CUresult (*GetIdFn)(CUcontext, unsigned long long*);
    static GetCurrentFn get_current = nullptr;
    static GetIdFn get_id = nullptr;
    if (!get_current || !get_id) {
        void* a = nullptr;
        void* b = nullptr;
        cudaDriverEntryPointQueryResult qa, qb;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &a, cudaEnableDefault, &qa) != cudaSuccess ||
            qa != cudaDriverEntryPointSuccess ||
            cudaGetDriverEntryPoint("cuCtxGetId", &b, cudaEnableDefault, &qb) != cudaSuccess ||
            qb != cudaDriverEntryPointSuccess)
            return 0;
        get_current = reinterpret_cast<GetCurrentFn>(a);
        get_id = reinterpret_cast<GetIdFn>(b);
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (get_current(&ctx) != CUDA_SUCCESS || !ctx) return 0;
    if (get_id(ctx, &id) != CUDA_SUCCESS) return 0;
    return id;
}

// Device address of the scratch array for the current device (set-up on the
// first call per device; nullptr and *status set on failure).  The address
// is cached with the id of the context it was resolved in: after a device
// reset the module is loaded again in a new context, and the first call
// there resolves the address afresh.
uint64_t* noalloc_scratch(uint32_t* status) {
    static std::mutex mu;
    static uint64_t* addr[kMaxDevices] = {};
    static unsigned long long ctx_id[kMaxDevices] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        *status = DH_ERR_CUDA;
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    const unsigned long long id = current_context_id();
    if (!addr[dev] || id == 0 || id != ctx_id[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_noalloc_argmax_scratch) != cudaSuccess || !p) {
            *status = DH_ERR_CUDA;
            return nullptr;
        }
        addr[dev] = static_cast<uint64_t*>(p);
        ctx_id[dev] = current_context_id();  // the lookup made the context current
    }
    return addr[dev];
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

uint32_t dh_philox4x32_10(const uint32_t* counters, const uint32_t* keys, uint32_t* out,
                          uint32_t count, void* stream) {
    if (!counters || !keys || !out) return DH_ERR_NULL_POINTER;
    if (count == 0) return DH_OK;
    philox_batch_kernel<<<(count + 255) / 256, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        counters, keys, out, count);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_gumbel_q10(const uint32_t* words, int32_t* scores, uint32_t count, void* stream) {
    if (!words || !scores) return DH_ERR_NULL_POINTER;
    if (count == 0) return DH_OK;
    const uint32_t blocks = min((count + 255) / 256, 4u * kNumSMs);
    gumbel_batch_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(words, scores,
                                                                              count);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

static uint32_t stream_common(void* out, bool scores, uint32_t positions, uint32_t vocab,
                              uint32_t eval_id, uint32_t stream_id, uint32_t seed_lo,
                              uint32_t seed_hi, void* stream) {
    if (positions == 0 || positions > 64) return DH_RNG_INVALID_POSITION_COUNT;
    if (vocab == 0 || vocab > 65535) return DH_RNG_INVALID_VOCABULARY_SIZE;
    if (!out) return DH_ERR_NULL_POINTER;
    const uint64_t total = static_cast<uint64_t>((vocab + 3) / 4) * positions;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((total + 255) / 256, 4ull * kNumSMs));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (scores)
        philox_stream_kernel<true><<<blocks, 256, 0, st>>>(out, positions, vocab, eval_id,
                                                           stream_id, seed_lo, seed_hi);
    else
        philox_stream_kernel<false><<<blocks, 256, 0, st>>>(out, positions, vocab, eval_id,
                                                            stream_id, seed_lo, seed_hi);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_philox_word_stream(uint32_t* out, uint32_t position_count, uint32_t vocabulary_size,
                               uint32_t evaluation_id, uint32_t stream_id, uint32_t seed_low,
                               uint32_t seed_high, void* stream) {
    return stream_common(out, false, position_count, vocabulary_size, evaluation_id, stream_id,
                         seed_low, seed_high, stream);
}

uint32_t dh_philox_gumbel_stream(int32_t* out, uint32_t position_count, uint32_t vocabulary_size,
                                 uint32_t evaluation_id, uint32_t stream_id, uint32_t seed_low,
                                 uint32_t seed_high, void* stream) {
    return stream_common(out, true, position_count, vocabulary_size, evaluation_id, stream_id,
                         seed_low, seed_high, stream);
}

size_t dh_noisy_argmax_workspace_size(uint32_t rows, uint32_t vocabulary_size) {
    return static_cast<size_t>(rows) * argmax_chunks(vocabulary_size) * sizeof(uint64_t);
}

uint32_t dh_noisy_argmax_f32(const float* logits, uint64_t row_stride, uint32_t rows,
                             uint32_t vocabulary_size, uint32_t mask_token_id,
                             const uint32_t* row_position, const uint32_t* row_key_hi,
                             const uint32_t* row_eval, uint32_t key_lo, uint32_t stream_id,
                             int32_t* out_ids, int32_t* out_scores, void* workspace,
                             size_t workspace_bytes, void* stream) {
    if (rows == 0 || rows > 65535u * 16u) return DH_RNG_INVALID_POSITION_COUNT;
    if (vocabulary_size == 0 || vocabulary_size > 65535 || mask_token_id >= vocabulary_size)
        return DH_RNG_INVALID_VOCABULARY_SIZE;
    if (!logits || !out_ids || !workspace) return DH_ERR_NULL_POINTER;
    if (row_stride < vocabulary_size) return DH_ERR_INVALID_ARGUMENT;
    if (rows > 65535u) return DH_ERR_UNSUPPORTED_SHAPE;
    if (workspace_bytes < dh_noisy_argmax_workspace_size(rows, vocabulary_size))
        return DH_ERR_WORKSPACE;
    ArgmaxRows a{logits, row_stride, rows, vocabulary_size, mask_token_id, row_position,
                 row_key_hi, row_eval, key_lo, stream_id, 0u, 0u, nullptr, nullptr};
    return launch_argmax(a, true, kFinalizeIds, out_ids, out_scores, nullptr, workspace,
                         static_cast<cudaStream_t>(stream));
}

// Same computation as dh_noisy_argmax_f32 without a caller workspace: for
// callers that cannot allocate device memory (see the header).  Calls that run
// at the same time on one GPU share the scratch array and race; serialise
// them (one stream, or events).  Nothing in the array needs to start at zero:
// each call writes every partial slot it later reads.
uint32_t dh_noisy_argmax_f32_noalloc(const float* logits, uint64_t row_stride, uint32_t rows,
                                     uint32_t vocabulary_size, uint32_t mask_token_id,
                                     const uint32_t* row_position, const uint32_t* row_key_hi,
                                     const uint32_t* row_eval, uint32_t key_lo, uint32_t stream_id,
                                     int32_t* out_ids, int32_t* out_scores, void* stream) {
    if (rows == 0 || rows > 65535u * 16u) return DH_RNG_INVALID_POSITION_COUNT;
    if (vocabulary_size == 0 || vocabulary_size > 65535 || mask_token_id >= vocabulary_size)
        return DH_RNG_INVALID_VOCABULARY_SIZE;
    if (!logits || !out_ids) return DH_ERR_NULL_POINTER;
    if (row_stride < vocabulary_size) return DH_ERR_INVALID_ARGUMENT;
    if (rows > 65535u) return DH_ERR_UNSUPPORTED_SHAPE;
    if (static_cast<uint64_t>(rows) * argmax_chunks(vocabulary_size) > kNoAllocScratchWords)
        return DH_ERR_SCRATCH_LIMIT;
    uint32_t status = DH_OK;
    uint64_t* scratch = noalloc_scratch(&status);
    if (!scratch) return status;
    ArgmaxRows a{logits, row_stride, rows, vocabulary_size, mask_token_id, row_position,
                 row_key_hi, row_eval, key_lo, stream_id, 0u, 0u, nullptr, nullptr};
    return launch_argmax(a, true, kFinalizeIds, out_ids, out_scores, nullptr, scratch,
                         static_cast<cudaStream_t>(stream));
}

uint32_t dh_greedy_argmax_f32(const float* logits, uint64_t row_stride, uint32_t rows,
                              uint32_t vocabulary_size, uint32_t mask_token_id, int32_t* out_ids,
                              void* workspace, size_t workspace_bytes, void* stream) {
    if (rows == 0) return DH_RNG_INVALID_POSITION_COUNT;
    if (vocabulary_size == 0 || vocabulary_size > 65535 || mask_token_id >= vocabulary_size)
        return DH_RNG_INVALID_VOCABULARY_SIZE;
    if (!logits || !out_ids || !workspace) return DH_ERR_NULL_POINTER;
    if (row_stride < vocabulary_size) return DH_ERR_INVALID_ARGUMENT;
    if (rows > 65535u) return DH_ERR_UNSUPPORTED_SHAPE;
    if (workspace_bytes < dh_noisy_argmax_workspace_size(rows, vocabulary_size))
        return DH_ERR_WORKSPACE;
    ArgmaxRows a{logits, row_stride, rows, vocabulary_size, mask_token_id, nullptr, nullptr,
                 nullptr, 0u, 0u, 0u, 0u, nullptr, nullptr};
    return launch_argmax(a, false, kFinalizeIds, out_ids, nullptr, nullptr, workspace,
                         static_cast<cudaStream_t>(stream));
}

uint32_t dh_candidate_reveal(uint16_t* tokens, const uint16_t* candidates, uint64_t* active,
                             uint64_t* valid, const uint32_t* words, uint64_t threshold_q32,
                             uint32_t positions, uint32_t sequences, uint64_t* results,
                             void* stream) {
    if (positions == 0) return DH_CAND_INVALID_POSITION_COUNT;
    if (threshold_q32 > DH_REVEAL_PROBABILITY_ONE_Q32) return DH_CAND_INVALID_THRESHOLD;
    if (!tokens || !candidates || !active || !valid || !words || !results)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0) return DH_OK;
    reveal_kernel<uint16_t, false><<<sequences, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        tokens, candidates, active, valid, words, threshold_q32, positions, results, nullptr,
        nullptr, 0u, 0u, nullptr);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_sampler_init(const int32_t* input_ids, uint32_t sequences, uint32_t positions,
                         uint32_t mask_token_id, uint32_t steps, int32_t* tokens,
                         uint16_t* candidates, uint64_t* active, uint64_t* valid,
                         uint32_t* eval_id, int32_t* counters, void* stream) {
    if (positions == 0) return DH_CAND_INVALID_POSITION_COUNT;
    if (!input_ids || !tokens || !candidates || !active || !valid || !eval_id || !counters)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0) return DH_ERR_INVALID_ARGUMENT;
    sampler_init_kernel<<<sequences, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        input_ids, sequences, positions, mask_token_id, steps, tokens, candidates, active, valid,
        eval_id, counters);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

size_t dh_sampler_workspace_size(uint32_t sequences, uint32_t positions,
                                 uint32_t vocabulary_size) {
    const size_t rows = static_cast<size_t>(sequences) * positions;
    const size_t refill = ((static_cast<size_t>(sequences) * 4 + 255) / 256) * 256;
    return refill + rows * argmax_chunks(vocabulary_size) * sizeof(uint64_t);
}

uint32_t dh_sampler_transition_f32(const float* logits, uint32_t sequences, uint32_t positions,
                                   uint32_t vocabulary_size, uint32_t mask_token_id,
                                   uint32_t seed, uint32_t step, uint32_t steps,
                                   uint64_t threshold_q32, int32_t* tokens, uint16_t* candidates,
                                   uint64_t* active, uint64_t* valid, uint32_t* eval_id,
                                   int32_t* counters, void* workspace, size_t workspace_bytes,
                                   void* stream) {
    if (positions == 0) return DH_CAND_INVALID_POSITION_COUNT;
    if (threshold_q32 > DH_REVEAL_PROBABILITY_ONE_Q32) return DH_CAND_INVALID_THRESHOLD;
    if (vocabulary_size == 0 || vocabulary_size > 65535 || mask_token_id >= vocabulary_size)
        return DH_ERR_INVALID_ARGUMENT;
    if (!logits || !tokens || !candidates || !active || !valid || !eval_id || !counters ||
        !workspace)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0 || step >= steps) return DH_ERR_INVALID_ARGUMENT;
    const uint64_t rows = static_cast<uint64_t>(sequences) * positions;
    if (rows > 65535u) return DH_ERR_UNSUPPORTED_SHAPE;
    if (workspace_bytes < dh_sampler_workspace_size(sequences, positions, vocabulary_size))
        return DH_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint32_t* refill = static_cast<uint32_t*>(workspace);
    void* partial = static_cast<char*>(workspace) +
                    ((static_cast<size_t>(sequences) * 4 + 255) / 256) * 256;
    sampler_plan_kernel<<<(sequences + 7) / 8, 256, 0, st>>>(active, valid, sequences, positions,
                                                              step, refill, counters);
    DH_LAUNCH_CHECK();
    // Refill: candidate of every row of a refilling sequence, counter
    // (v/4, position, step, 0), key (seed, sequence).
    ArgmaxRows a{logits, vocabulary_size, static_cast<uint32_t>(rows), vocabulary_size,
                 mask_token_id, nullptr, nullptr, nullptr, seed, 0u, positions, step, refill,
                 nullptr};
    uint32_t status = launch_argmax(a, true, kFinalizeCandidates, nullptr, nullptr, candidates,
                                    partial, st);
    if (status != DH_OK) return status;
    reveal_kernel<int32_t, true><<<sequences, 256, 0, st>>>(
        tokens, candidates, active, valid, nullptr, threshold_q32, positions, nullptr, refill,
        eval_id, seed, step, counters);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_sampler_finalize_f32(const float* logits, uint32_t sequences, uint32_t positions,
                                 uint32_t vocabulary_size, uint32_t mask_token_id,
                                 int32_t* tokens, uint64_t* active, void* workspace,
                                 size_t workspace_bytes, void* stream) {
    if (positions == 0) return DH_CAND_INVALID_POSITION_COUNT;
    if (vocabulary_size == 0 || vocabulary_size > 65535 || mask_token_id >= vocabulary_size)
        return DH_ERR_INVALID_ARGUMENT;
    if (!logits || !tokens || !active || !workspace) return DH_ERR_NULL_POINTER;
    if (positions % 64 != 0) return DH_ERR_UNSUPPORTED_SHAPE;
    const uint64_t rows = static_cast<uint64_t>(sequences) * positions;
    if (rows == 0 || rows > 65535u) return DH_ERR_UNSUPPORTED_SHAPE;
    if (workspace_bytes < dh_sampler_workspace_size(sequences, positions, vocabulary_size))
        return DH_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    void* partial = static_cast<char*>(workspace) +
                    ((static_cast<size_t>(sequences) * 4 + 255) / 256) * 256;
    // With positions a multiple of 64 the [B][W] bitmap is the flat row bitmap.
    ArgmaxRows a{logits, vocabulary_size, static_cast<uint32_t>(rows), vocabulary_size,
                 mask_token_id, nullptr, nullptr, nullptr, 0u, 0u, positions, 0u, nullptr,
                 active};
    uint32_t status = launch_argmax(a, false, kFinalizeGreedyCommit, tokens, nullptr, nullptr,
                                    partial, st);
    if (status != DH_OK) return status;
    const uint64_t words = rows / 64;
    clear_bitmap_kernel<<<static_cast<uint32_t>((words + 255) / 256), 256, 0, st>>>(active, words);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

}  // extern "C"
