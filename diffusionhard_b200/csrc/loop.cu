// loop.cu -- device side of the ddpm_cache / candidate-cache loop around the
// model (mdlm.py:1104-1218), with the selected-row head:
//
//   plan    per sequence: active count; a sequence whose canvas changed at
//           the previous transition refills its cache (needs a forward); the
//           forward runs (fwd_rows = B*L) iff some sequence refills.
//   select  reveal decision of every active position, word
//           philox((p/4, 0, k, 1), (seed, b))[p%4] < threshold_k, compacted
//           in position-major order into a row list with the row's noise
//           counter fields (position p, key_hi b, eval = transition of b's
//           last evaluation).
//   [head]  candidates for the selected rows only (head.cu)
//   commit  tokens <- candidates, clear active bits, mark changed sequences.
//
// Computing candidates only for the revealed rows is pathwise identical to
// drawing them for every row at evaluation time: the noise of (b, p, v) is a
// function of the counter only, and candidates of rows that do not reveal are
// discarded by the reference anyway (mdlm.py:1155-1174).
#include "dh_common.cuh"
#include "dh_philox.cuh"

#include <algorithm>

namespace dh {
namespace {

// Single CTA: B sequences x W bitmap words.  A sequence refills when it has
// masked positions and its canvas changed at the previous transition (every
// sequence with masked positions on the final pass).  Without a sequence
// list the forward covers the whole batch whenever one sequence refills
// (fwd_rows = B * L or 0); with one, seq_list[0 .. n) receives the refilling
// sequences in ascending order and fwd_rows = n * L, so the forward runs
// over those sequences only, packed together.
__global__ void __launch_bounds__(1024)
loop_plan_kernel(uint32_t B, uint32_t L, uint32_t step, uint32_t final_pass,
                 const uint64_t* __restrict__ active, uint32_t* __restrict__ need_eval,
                 uint32_t* __restrict__ eval_id, uint32_t* __restrict__ fwd_rows,
                 uint32_t* __restrict__ sel_count, int32_t* __restrict__ counters,
                 uint32_t* __restrict__ seq_list) {
    __shared__ uint32_t any_refill, total_active, listed;
    __shared__ uint32_t warp_base[32];
    if (threadIdx.x == 0) {
        any_refill = 0;
        total_active = 0;
        listed = 0;
        *sel_count = 0;
    }
    __syncthreads();
    const uint32_t W = (L + 63) / 64;
    const uint32_t warps = blockDim.x / 32;
    // rounds of `warps` sequences: warp i takes sequence round * warps + i,
    // so the list stays in ascending order
    for (uint32_t base = 0; base < B; base += warps) {
        const uint32_t b = base + warp_id();
        uint32_t refill = 0;
        if (b < B) {
            uint32_t cnt = 0;
            for (uint32_t w = lane_id(); w < W; w += 32) cnt += __popcll(active[static_cast<uint64_t>(b) * W + w]);
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xFFFFFFFFu, cnt, o);
            refill = (cnt > 0 && (final_pass || need_eval[b])) ? 1u : 0u;
            if (lane_id() == 0) {
                if (cnt) atomicAdd(&total_active, cnt);
                if (refill) {
                    any_refill = 1;
                    if (!final_pass) {
                        eval_id[b] = step;
                        need_eval[b] = 0;
                    }
                }
            }
        }
        if (seq_list) {
            if (lane_id() == 0) warp_base[warp_id()] = refill;
            __syncthreads();
            if (threadIdx.x == 0) {
                uint32_t run = listed;
                for (uint32_t i = 0; i < warps; ++i) {
                    const uint32_t f = warp_base[i];
                    warp_base[i] = run;
                    run += f;
                }
                listed = run;
            }
            __syncthreads();
            if (refill && lane_id() == 0) seq_list[warp_base[warp_id()]] = b;
            __syncthreads();
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        *fwd_rows = seq_list ? listed * L : (any_refill ? B * L : 0u);
        if (!final_pass) {
            counters[3 * step] = static_cast<int32_t>(total_active);
            counters[3 * step + 2] = static_cast<int32_t>(any_refill);
        }
    }
}

// One CTA compacts the revealed rows of the whole batch in position-major
// order (ballot + block scan, no atomics), so the row list is a deterministic
// function of the state: replicated ranks of the vocab-sharded head reduce
// their per-row results slot by slot.
__global__ void __launch_bounds__(1024)
loop_select_kernel(uint32_t B, uint32_t L, uint32_t step, uint32_t seed, uint32_t seq_offset,
                   uint32_t position_offset, uint64_t threshold, uint32_t final_pass, const uint64_t* __restrict__ active,
                   const uint32_t* __restrict__ eval_id, uint32_t* __restrict__ sel_rows,
                   uint32_t* __restrict__ sel_pos, uint32_t* __restrict__ sel_key,
                   uint32_t* __restrict__ sel_eval, uint32_t* __restrict__ sel_count) {
    __shared__ uint32_t warp_off[32];
    __shared__ uint32_t iter_total, base;
    const uint32_t W = (L + 63) / 64;
    const uint64_t total = static_cast<uint64_t>(B) * L;
    if (threadIdx.x == 0) base = 0;
    __syncthreads();
    for (uint64_t start = 0; start < total; start += blockDim.x) {
        const uint64_t idx = start + threadIdx.x;
        bool take = false;
        uint32_t b = 0, p = 0;
        if (idx < total) {
            b = static_cast<uint32_t>(idx / L);
            p = static_cast<uint32_t>(idx % L);
            const bool act = (active[static_cast<uint64_t>(b) * W + (p >> 6)] >> (p & 63u)) & 1ull;
            if (act) {
                if (final_pass) {
                    take = true;
                } else {
                    const uint32_t gp = position_offset + p;  // canvas position
                    Philox4 r = philox4x32_10(gp >> 2, 0u, step, 1u, seed, seq_offset + b);
                    take = static_cast<uint64_t>(philox_lane(r, gp & 3u)) < threshold;
                }
            }
        }
        const uint32_t mask = __ballot_sync(0xFFFFFFFFu, take);
        if (lane_id() == 0) warp_off[warp_id()] = __popc(mask);
        __syncthreads();
        if (warp_id() == 0) {
            const uint32_t nw = blockDim.x / 32;
            const uint32_t c = lane_id() < nw ? warp_off[lane_id()] : 0u;
            uint32_t inc = c;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xFFFFFFFFu, inc, o);
                if (lane_id() >= static_cast<uint32_t>(o)) inc += t;
            }
            if (lane_id() < nw) warp_off[lane_id()] = inc - c;
            if (lane_id() == 31) iter_total = inc;
        }
        __syncthreads();
        if (take) {
            const uint32_t slot = base + warp_off[warp_id()] + __popc(mask & ((1u << lane_id()) - 1u));
            sel_rows[slot] = b * L + p;
            sel_pos[slot] = position_offset + p;
            sel_key[slot] = seq_offset + b;
            sel_eval[slot] = eval_id[b];
        }
        __syncthreads();
        if (threadIdx.x == 0) base += iter_total;
        __syncthreads();
    }
    if (threadIdx.x == 0) *sel_count = base;
}

__global__ void loop_commit_kernel(uint32_t L, uint32_t step, uint32_t final_pass,
                                   const unsigned long long* __restrict__ packed,
                                   const uint32_t* __restrict__ sel_rows,
                                   const uint32_t* __restrict__ sel_count,
                                   int32_t* __restrict__ tokens, uint64_t* __restrict__ active,
                                   uint32_t* __restrict__ need_eval, int32_t* __restrict__ counters) {
    const uint32_t n = *sel_count;
    const uint32_t W = (L + 63) / 64;
    uint32_t mine = 0;
    for (uint32_t i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const uint32_t r = sel_rows[i];
        const uint32_t b = r / L, p = r % L;
        const unsigned long long pk = packed[i];
        tokens[r] = static_cast<int32_t>(pk == 0ull ? 0u : packed_id(pk));
        atomicAnd(reinterpret_cast<unsigned long long*>(active) + static_cast<uint64_t>(b) * W + (p >> 6),
                  ~(1ull << (p & 63u)));
        need_eval[b] = 1u;
        ++mine;
    }
    if (!final_pass) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) mine += __shfl_xor_sync(0xFFFFFFFFu, mine, o);
        if (lane_id() == 0 && mine) atomicAdd(&counters[3 * step + 1], static_cast<int32_t>(mine));
    }
}

__global__ void loop_init_kernel(const int32_t* __restrict__ input_ids, uint32_t L, uint32_t mask_id,
                                 uint32_t steps, int32_t* __restrict__ tokens,
                                 uint64_t* __restrict__ active, uint32_t* __restrict__ need_eval,
                                 uint32_t* __restrict__ eval_id, int32_t* __restrict__ counters) {
    const uint32_t b = blockIdx.x;
    const uint32_t W = (L + 63) / 64;
    for (uint32_t w = warp_id(); w < W; w += blockDim.x / 32) {
        uint32_t m[2];
#pragma unroll
        for (uint32_t h = 0; h < 2; ++h) {
            const uint32_t p = w * 64 + lane_id() + 32 * h;
            m[h] = 0;
            if (p < L) {
                const uint64_t i = static_cast<uint64_t>(b) * L + p;
                tokens[i] = input_ids[i];
                m[h] = static_cast<uint32_t>(input_ids[i]) == mask_id;
            }
        }
        const uint32_t lo = __ballot_sync(0xFFFFFFFFu, m[0]);
        const uint32_t hi = __ballot_sync(0xFFFFFFFFu, m[1]);
        if (lane_id() == 0) active[static_cast<uint64_t>(b) * W + w] = (static_cast<uint64_t>(hi) << 32) | lo;
    }
    if (threadIdx.x == 0) {
        need_eval[b] = 1u;
        eval_id[b] = 0u;
    }
    if (b == 0)
        for (uint32_t i = threadIdx.x; i < 3 * steps; i += blockDim.x) counters[i] = 0;
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

uint32_t dh_loop_init(const int32_t* input_ids, uint32_t sequences, uint32_t positions,
                      uint32_t mask_token_id, uint32_t steps, int32_t* tokens, uint64_t* active,
                      uint32_t* need_eval, uint32_t* eval_id, int32_t* counters, void* stream) {
    if (!input_ids || !tokens || !active || !need_eval || !eval_id || !counters)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0 || positions == 0) return DH_ERR_INVALID_ARGUMENT;
    loop_init_kernel<<<sequences, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        input_ids, positions, mask_token_id, steps, tokens, active, need_eval, eval_id, counters);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_loop_plan(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t steps,
                      uint32_t final_pass, const uint64_t* active, uint32_t* need_eval,
                      uint32_t* eval_id, uint32_t* fwd_rows, uint32_t* sel_count,
                      int32_t* counters, void* stream) {
    return dh_loop_plan_seqs(sequences, positions, step, steps, final_pass, active, need_eval, eval_id, fwd_rows,
                             sel_count, counters, nullptr, stream);
}

uint32_t dh_loop_plan_seqs(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t steps,
                           uint32_t final_pass, const uint64_t* active, uint32_t* need_eval,
                           uint32_t* eval_id, uint32_t* fwd_rows, uint32_t* sel_count,
                           int32_t* counters, uint32_t* seq_list, void* stream) {
    if (!active || !need_eval || !eval_id || !fwd_rows || !sel_count || !counters)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0 || positions == 0 || (!final_pass && step >= steps))
        return DH_ERR_INVALID_ARGUMENT;
    if (static_cast<uint64_t>(sequences) * positions > 0xFFFFFFFFull) return DH_ERR_UNSUPPORTED_SHAPE;
    loop_plan_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
        sequences, positions, step, final_pass, active, need_eval, eval_id, fwd_rows, sel_count,
        counters, seq_list);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_loop_select(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t seed,
                        uint32_t seq_offset, uint32_t position_offset, uint64_t threshold_q32, uint32_t final_pass, const uint64_t* active,
                        const uint32_t* eval_id, uint32_t* sel_rows, uint32_t* sel_pos,
                        uint32_t* sel_key, uint32_t* sel_eval, uint32_t* sel_count, void* stream) {
    if (threshold_q32 > DH_REVEAL_PROBABILITY_ONE_Q32) return DH_CAND_INVALID_THRESHOLD;
    if (!active || !eval_id || !sel_rows || !sel_pos || !sel_key || !sel_eval || !sel_count)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0 || positions == 0) return DH_ERR_INVALID_ARGUMENT;
    loop_select_kernel<<<1, 1024, 0, static_cast<cudaStream_t>(stream)>>>(
        sequences, positions, step, seed, seq_offset, position_offset, threshold_q32, final_pass, active,
        eval_id,
        sel_rows, sel_pos, sel_key, sel_eval, sel_count);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

uint32_t dh_loop_commit(uint32_t sequences, uint32_t positions, uint32_t step, uint32_t steps,
                        uint32_t final_pass, const uint64_t* packed, const uint32_t* sel_rows,
                        const uint32_t* sel_count, int32_t* tokens, uint64_t* active,
                        uint32_t* need_eval, int32_t* counters, void* stream) {
    if (!packed || !sel_rows || !sel_count || !tokens || !active || !need_eval || !counters)
        return DH_ERR_NULL_POINTER;
    if (sequences == 0 || positions == 0 || (!final_pass && step >= steps))
        return DH_ERR_INVALID_ARGUMENT;
    const uint64_t rows = static_cast<uint64_t>(sequences) * positions;
    const uint32_t blocks = static_cast<uint32_t>(std::min<uint64_t>((rows + 255) / 256, 4ull * kNumSMs));
    loop_commit_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        positions, step, final_pass, reinterpret_cast<const unsigned long long*>(packed), sel_rows,
        sel_count, tokens, active, need_eval, counters);
    DH_LAUNCH_CHECK();
    return DH_OK;
}

}  // extern "C"
