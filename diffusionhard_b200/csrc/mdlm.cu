// mdlm.cu -- composite entry points of the MDLM path, enqueued from C++ on
// one stream with no host synchronisation:
//
//   dh_ddit_forward        the whole W8A8 DDiT forward (embedding gather, then
//                          per block LN+quant -> QKV+rotary -> attention ->
//                          quant -> out+residual -> LN+quant -> up+GELU ->
//                          quant -> down+residual), the folded forward of
//                          hardware_package.folded_mdlm_forward
//                          (hardware_package.py:195-289);
//   dh_sample_loop         the whole candidate-cache generation
//                          (mdlm._run_ddpm_candidate_cache_sampler,
//                          mdlm.py:1104-1218): per transition plan -> forward
//                          (skipped on the device when no sequence refills)
//                          -> reveal select -> final LN + quant of the
//                          revealed rows -> fused head + Philox-Gumbel argmax
//                          -> [vocab-shard reduce] -> commit, then the greedy
//                          final pass;
//   dh_vocab_shard_reduce  the (max score, lowest id) merge of the packed
//                          per-row head results over a caller's NCCL
//                          communicator (ordered_noisy_argmax_reducer.sv:106-133).
//
// They call the per-kernel entry points of the other files, so they launch
// exactly the kernels a host that orchestrates those entry points itself
// would.  Arguments are checked before anything is enqueued; the caller
// owns every buffer (workspace sizes from the *_workspace_size queries).
#include <dlfcn.h>
#include <nccl.h>

#include <mutex>

#include "dh_common.cuh"

namespace dh {
namespace {

constexpr uint32_t kHidden = 768, kQKV = 2304, kMlp = 3072, kHeadsN = 12, kHeadDim = 64;

inline size_t align256(size_t v) { return (v + 255) & ~static_cast<size_t>(255); }

// Offsets of the workspace regions (256-byte aligned), forward first; the
// loop adds the residual stream, the head input and the loop state.
struct Layout {
    size_t act_q, act_scale, q, k, vt, attn, mlp, row_amax, fwd_end;
    size_t x, xs, head_q, head_scale, packed, active, need_eval, eval_id, fwd_rows, sel_count;
    size_t sel_rows, sel_pos, sel_key, sel_eval, seq_list, head_all, head_all_scale, loop_end;
};

Layout layout(uint32_t B, uint32_t L) {
    const size_t M = static_cast<size_t>(B) * L;
    const size_t bhl = static_cast<size_t>(B) * kHeadsN * L * kHeadDim;
    Layout o{};
    size_t at = 0;
    auto take = [&](size_t bytes) {
        const size_t here = at;
        at = align256(at + bytes);
        return here;
    };
    o.act_q = take(M * kMlp);
    o.act_scale = take(M * 4);
    o.q = take(bhl * 2);
    o.k = take(bhl * 2);
    o.vt = take(bhl * 2);
    o.attn = take(M * kHidden * 2);
    o.mlp = take(M * kMlp * 2);
    o.row_amax = take(M * 4);
    o.fwd_end = at;
    o.x = take(M * kHidden * 4);
    o.xs = take(M * kHidden * 4);
    o.head_q = take(M * kHidden);
    o.head_scale = take(M * 4);
    o.packed = take(M * 8);
    o.active = take(static_cast<size_t>(B) * ((L + 63) / 64) * 8);
    o.need_eval = take(static_cast<size_t>(B) * 4);
    o.eval_id = take(static_cast<size_t>(B) * 4);
    o.fwd_rows = take(4);
    o.sel_count = take(4);
    o.sel_rows = take(M * 4);
    o.sel_pos = take(M * 4);
    o.sel_key = take(M * 4);
    o.sel_eval = take(M * 4);
    o.seq_list = take(static_cast<size_t>(B) * 4);
    o.head_all = take(M * kHidden);
    o.head_all_scale = take(M * 4);
    o.loop_end = at;
    return o;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

uint32_t check_linear(const dh_linear_weights& l, bool needs_bias) {
    if (!l.weight || !l.w_scale || !l.smooth || !l.inv_smooth || (needs_bias && !l.bias)) return DH_ERR_NULL_POINTER;
    if (!aligned16(l.weight) || !aligned16(l.w_scale) || !aligned16(l.smooth) || !aligned16(l.inv_smooth) ||
        (l.bias && !aligned16(l.bias)))
        return DH_ERR_ALIGNMENT;
    return DH_OK;
}

// Everything the forward reads, checked before the first launch.
uint32_t check_model(const dh_mdlm_weights* w, uint32_t B, uint32_t L) {
    if (!w) return DH_ERR_NULL_POINTER;
    if (w->blocks == 0 || B == 0 || L == 0 || w->vocabulary_size == 0 || w->mask_token_id >= w->vocabulary_size)
        return DH_ERR_INVALID_ARGUMENT;
    if (L % 32 != 0 || L > w->max_positions) return DH_ERR_UNSUPPORTED_SHAPE;
    if (static_cast<uint64_t>(B) * L > (1ull << 31) / kMlp) return DH_ERR_UNSUPPORTED_SHAPE;
    if (!w->embedding || !w->rope_cos || !w->rope_sin || !w->block_linears) return DH_ERR_NULL_POINTER;
    if (!aligned16(w->embedding) || !aligned16(w->rope_cos) || !aligned16(w->rope_sin)) return DH_ERR_ALIGNMENT;
    for (uint32_t i = 0; i < w->blocks; ++i) {
        const dh_linear_weights* bl = w->block_linears + 4 * i;
        uint32_t st;
        if ((st = check_linear(bl[0], true)) != DH_OK || (st = check_linear(bl[1], false)) != DH_OK ||
            (st = check_linear(bl[2], true)) != DH_OK || (st = check_linear(bl[3], false)) != DH_OK)
            return st;
    }
    return DH_OK;
}

#define DH_TRY(expr)                       \
    do {                                   \
        const uint32_t _s = (expr);        \
        if (_s != DH_OK) return _s;        \
    } while (0)

template <class T>
T* at(void* base, size_t off) {
    return reinterpret_cast<T*>(static_cast<uint8_t*>(base) + off);
}

// The forward over B x L rows of `tokens`, residual stream into x.  run_rows:
// device word, the launches process only its first *run_rows rows (0: none).
// seq_list (device, may be NULL): the rows are the packed positions of the
// listed sequences of `tokens` (the sequences that need a forward).
uint32_t enqueue_forward(const dh_mdlm_weights* w, const int32_t* tokens, uint32_t B, uint32_t L, float* x,
                         void* ws, const Layout& o, const uint32_t* run_rows, void* s,
                         const uint32_t* seq_list = nullptr, bool stop_at_last_attention = false) {
    const uint32_t M = B * L;
    int8_t* act_q = at<int8_t>(ws, o.act_q);
    float* act_scale = at<float>(ws, o.act_scale);
    void* q = at<void>(ws, o.q);
    void* k = at<void>(ws, o.k);
    void* vt = at<void>(ws, o.vt);
    void* attn = at<void>(ws, o.attn);
    void* mlp = at<void>(ws, o.mlp);
    uint32_t* row_amax = at<uint32_t>(ws, o.row_amax);
    if (seq_list)
        DH_TRY(dh_embed_gather_seqs(tokens, seq_list, L, w->embedding, x, M, w->vocabulary_size, run_rows, s));
    else
        DH_TRY(dh_embed_gather(tokens, w->embedding, x, M, w->vocabulary_size, run_rows, s));
    for (uint32_t i = 0; i < w->blocks; ++i) {
        const dh_linear_weights& qkv = w->block_linears[4 * i];
        const dh_linear_weights& out = w->block_linears[4 * i + 1];
        const dh_linear_weights& up = w->block_linears[4 * i + 2];
        const dh_linear_weights& down = w->block_linears[4 * i + 3];
        DH_TRY(dh_ln_smooth_quant(x, qkv.smooth, qkv.inv_smooth, act_q, act_scale, M, nullptr, nullptr, run_rows, s));
        DH_TRY(dh_gemm_qkv_rope(act_q, act_scale, qkv.weight, qkv.w_scale, qkv.bias, w->rope_cos, w->rope_sin,
                                out.inv_smooth, M, L, 0, L, 0, q, k, vt, run_rows, s));
        DH_TRY(dh_attention(q, k, vt, attn, B, L, L, L, run_rows, s));
        // the loop finishes the last block for the revealed rows only
        // (enqueue_last_block_rows): x keeps the input of the last block and
        // attn its attention output, for every row
        if (stop_at_last_attention && i + 1 == w->blocks) break;
        DH_TRY(dh_quant_rows_bf16(attn, nullptr, nullptr, act_q, act_scale, M, kHidden, run_rows, s));
        DH_TRY(dh_gemm_residual(act_q, act_scale, out.weight, out.w_scale, out.bias, x, M, kHidden, kHidden,
                                run_rows, s));
        DH_TRY(dh_ln_smooth_quant(x, up.smooth, up.inv_smooth, act_q, act_scale, M, nullptr, nullptr, run_rows, s));
        DH_TRY(dh_gemm_gelu(act_q, act_scale, up.weight, up.w_scale, up.bias, down.inv_smooth, mlp, row_amax, M,
                            kMlp, kHidden, run_rows, s));
        DH_TRY(dh_quant_rows_bf16_amax(mlp, row_amax, act_q, act_scale, M, kMlp, run_rows, s));
        DH_TRY(dh_gemm_residual(act_q, act_scale, down.weight, down.w_scale, down.bias, x, M, kHidden, kMlp,
                                run_rows, s));
    }
    return DH_OK;
}

// The rest of the last block (requant, attention-out + residual, LayerNorm,
// MLP + residual) and the final LayerNorm + head quantisation, for the
// *sel_count rows listed in sel_rows only: the head reads nothing else, and
// every one of these steps is row-wise, so the rows get the bits the whole-
// batch block would give them.  Inputs: x = the residual stream entering
// the last block and attn = its attention output, both for every row (the
// last forward's, also when this transition ran none).  The rows are
// gathered into xs and q (free after the attention); head_q / head_scale
// receive the head's int8 input rows 0 .. *sel_count.
uint32_t enqueue_last_block_rows(const dh_mdlm_weights* w, uint32_t B, uint32_t L, void* ws, const Layout& o,
                                 const uint32_t* sel_rows, const uint32_t* sel_count, void* s) {
    const uint32_t M = B * L;
    const uint32_t i = w->blocks - 1;
    const dh_linear_weights& out = w->block_linears[4 * i + 1];
    const dh_linear_weights& up = w->block_linears[4 * i + 2];
    const dh_linear_weights& down = w->block_linears[4 * i + 3];
    const float* x = at<float>(ws, o.x);
    float* xs = at<float>(ws, o.xs);
    const void* attn = at<void>(ws, o.attn);
    void* attn_rows = at<void>(ws, o.q);
    int8_t* act_q = at<int8_t>(ws, o.act_q);
    float* act_scale = at<float>(ws, o.act_scale);
    void* mlp = at<void>(ws, o.mlp);
    uint32_t* row_amax = at<uint32_t>(ws, o.row_amax);
    DH_TRY(dh_gather_rows(x, kHidden * 4, sel_rows, sel_count, M, xs, s));
    DH_TRY(dh_gather_rows(attn, kHidden * 2, sel_rows, sel_count, M, attn_rows, s));
    DH_TRY(dh_quant_rows_bf16(attn_rows, nullptr, nullptr, act_q, act_scale, M, kHidden, sel_count, s));
    DH_TRY(dh_gemm_residual(act_q, act_scale, out.weight, out.w_scale, out.bias, xs, M, kHidden, kHidden, sel_count,
                            s));
    DH_TRY(dh_ln_smooth_quant(xs, up.smooth, up.inv_smooth, act_q, act_scale, M, nullptr, nullptr, sel_count, s));
    DH_TRY(dh_gemm_gelu(act_q, act_scale, up.weight, up.w_scale, up.bias, down.inv_smooth, mlp, row_amax, M, kMlp,
                        kHidden, sel_count, s));
    DH_TRY(dh_quant_rows_bf16_amax(mlp, row_amax, act_q, act_scale, M, kMlp, sel_count, s));
    DH_TRY(dh_gemm_residual(act_q, act_scale, down.weight, down.w_scale, down.bias, xs, M, kHidden, kMlp, sel_count,
                            s));
    DH_TRY(dh_ln_smooth_quant(xs, w->head.smooth, w->head.inv_smooth, at<int8_t>(ws, o.head_q),
                              at<float>(ws, o.head_scale), M, nullptr, nullptr, sel_count, s));
    return DH_OK;
}

// ncclAllReduce of the NCCL library the process has loaded (the one that
// made the caller's communicator), resolved at the first call.
typedef ncclResult_t (*AllReduceFn)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                    cudaStream_t);

AllReduceFn nccl_all_reduce() {
    static std::once_flag once;
    static AllReduceFn fn = nullptr;
    std::call_once(once, [] {
        void* h = dlopen("libnccl.so.2", RTLD_LAZY | RTLD_NOLOAD);
        void* p = h ? dlsym(h, "ncclAllReduce") : nullptr;
        if (!p) p = dlsym(RTLD_DEFAULT, "ncclAllReduce");
        fn = reinterpret_cast<AllReduceFn>(p);
    });
    return fn;
}

}  // namespace
}  // namespace dh

using namespace dh;

extern "C" {

size_t dh_ddit_forward_workspace_size(uint32_t sequences, uint32_t positions) {
    return layout(sequences, positions).fwd_end;
}

uint32_t dh_ddit_forward(const dh_mdlm_weights* weights, const int32_t* tokens, uint32_t sequences,
                         uint32_t positions, float* x, void* workspace, size_t workspace_bytes,
                         const uint32_t* run_rows, void* stream) {
    DH_TRY(check_model(weights, sequences, positions));
    if (!tokens || !x || !workspace) return DH_ERR_NULL_POINTER;
    if (!aligned16(x) || (reinterpret_cast<uintptr_t>(workspace) & 255u)) return DH_ERR_ALIGNMENT;
    const Layout o = layout(sequences, positions);
    if (workspace_bytes < o.fwd_end) return DH_ERR_WORKSPACE;
    // the MLP row-amax words start at 0 (each quantiser launch clears them again)
    if (cudaMemsetAsync(at<uint8_t>(workspace, o.row_amax), 0, static_cast<size_t>(sequences) * positions * 4,
                        static_cast<cudaStream_t>(stream)) != cudaSuccess)
        return DH_ERR_CUDA;
    return enqueue_forward(weights, tokens, sequences, positions, x, workspace, o, run_rows, stream);
}

uint32_t dh_vocab_shard_reduce(void* nccl_comm, uint64_t* packed, uint64_t count, void* stream) {
    if (!nccl_comm || !packed) return DH_ERR_NULL_POINTER;
    if (count == 0) return DH_OK;
    AllReduceFn fn = nccl_all_reduce();
    if (!fn) return DH_ERR_NCCL;
    // packed = (score ^ 0x80000000) << 32 | ~id: the unsigned order is the
    // (score, lower id) order, so an unsigned MAX merges the shards
    if (fn(packed, packed, count, ncclUint64, ncclMax, static_cast<ncclComm_t>(nccl_comm),
           static_cast<cudaStream_t>(stream)) != ncclSuccess)
        return DH_ERR_NCCL;
    return DH_OK;
}

size_t dh_sample_loop_workspace_size(uint32_t sequences, uint32_t positions) {
    return layout(sequences, positions).loop_end;
}

uint32_t dh_sample_loop(const dh_mdlm_weights* weights, const int32_t* input_ids, int32_t* tokens,
                        uint32_t sequences, uint32_t positions, uint32_t steps, const uint64_t* thresholds_q32,
                        uint32_t seed, uint32_t seq_offset, int32_t* counters, void* nccl_comm, uint32_t compact,
                        void* workspace, size_t workspace_bytes, void* stream) {
    DH_TRY(check_model(weights, sequences, positions));
    const dh_mdlm_weights* w = weights;
    if (!input_ids || !tokens || !thresholds_q32 || !counters || !workspace) return DH_ERR_NULL_POINTER;
    if (steps == 0) return DH_ERR_INVALID_ARGUMENT;
    for (uint32_t k = 0; k < steps; ++k)
        if (thresholds_q32[k] > DH_REVEAL_PROBABILITY_ONE_Q32) return DH_CAND_INVALID_THRESHOLD;
    if (!w->head.weight || !w->head.w_scale || !w->head.bias || !w->head.smooth) return DH_ERR_NULL_POINTER;
    if (w->head_rows == 0 || w->head_vocab_offset % 4 != 0 ||
        static_cast<uint64_t>(w->head_vocab_offset) + w->head_rows > w->vocabulary_size)
        return DH_ERR_INVALID_ARGUMENT;
    if (reinterpret_cast<uintptr_t>(workspace) & 255u) return DH_ERR_ALIGNMENT;
    const Layout o = layout(sequences, positions);
    if (workspace_bytes < o.loop_end) return DH_ERR_WORKSPACE;
    if (nccl_comm && !nccl_all_reduce()) return DH_ERR_NCCL;

    const uint32_t B = sequences, L = positions, M = B * L;
    float* x = at<float>(workspace, o.x);
    int8_t* head_q = at<int8_t>(workspace, o.head_q);
    float* head_scale = at<float>(workspace, o.head_scale);
    uint64_t* packed = at<uint64_t>(workspace, o.packed);
    uint64_t* active = at<uint64_t>(workspace, o.active);
    uint32_t* need_eval = at<uint32_t>(workspace, o.need_eval);
    uint32_t* eval_id = at<uint32_t>(workspace, o.eval_id);
    uint32_t* fwd_rows = at<uint32_t>(workspace, o.fwd_rows);
    uint32_t* sel_count = at<uint32_t>(workspace, o.sel_count);
    uint32_t* sel_rows = at<uint32_t>(workspace, o.sel_rows);
    uint32_t* sel_pos = at<uint32_t>(workspace, o.sel_pos);
    uint32_t* sel_key = at<uint32_t>(workspace, o.sel_key);
    uint32_t* sel_eval = at<uint32_t>(workspace, o.sel_eval);
    uint32_t* seq_list = compact ? at<uint32_t>(workspace, o.seq_list) : nullptr;
    int8_t* head_all = at<int8_t>(workspace, o.head_all);
    float* head_all_scale = at<float>(workspace, o.head_all_scale);
    void* s = stream;
    if (cudaMemsetAsync(at<uint8_t>(workspace, o.row_amax), 0, static_cast<size_t>(M) * 4,
                        static_cast<cudaStream_t>(s)) != cudaSuccess)
        return DH_ERR_CUDA;
    DH_TRY(dh_loop_init(input_ids, B, L, w->mask_token_id, steps, tokens, active, need_eval, eval_id, counters, s));
    for (uint32_t t = 0; t <= steps; ++t) {
        const uint32_t final_pass = t == steps ? 1u : 0u;
        const uint32_t k = final_pass ? steps - 1 : t;
        DH_TRY(dh_loop_plan_seqs(B, L, k, steps, final_pass, active, need_eval, eval_id, fwd_rows, sel_count,
                                 counters, seq_list, s));
        DH_TRY(enqueue_forward(w, tokens, B, L, x, workspace, o, fwd_rows, s, seq_list, seq_list == nullptr));
        if (seq_list)  // every refilled row's head input, kept per sequence until its next forward
            DH_TRY(dh_ln_smooth_quant_scatter(x, w->head.smooth, w->head.inv_smooth, head_all, head_all_scale, M,
                                              seq_list, L, fwd_rows, s));
        DH_TRY(dh_loop_select(B, L, k, seed, seq_offset, 0, final_pass ? 0 : thresholds_q32[t], final_pass, active,
                              eval_id, sel_rows, sel_pos, sel_key, sel_eval, sel_count, s));
        if (seq_list)
            DH_TRY(dh_gather_rows_i8(head_all, head_all_scale, sel_rows, sel_count, M, head_q, head_scale, s));
        else
            DH_TRY(enqueue_last_block_rows(w, B, L, workspace, o, sel_rows, sel_count, s));
        DH_TRY(dh_head_argmax_i8(head_q, kHidden, w->head.weight, kHidden, M, sel_count, kHidden, w->head_rows,
                                 w->head_vocab_offset, w->mask_token_id, final_pass ? 2u : 1u, head_scale,
                                 w->head.w_scale, w->head.bias, nullptr, nullptr, nullptr, sel_pos, sel_key, sel_eval,
                                 0, seed, 0, packed, nullptr, nullptr, s));
        if (nccl_comm) DH_TRY(dh_vocab_shard_reduce(nccl_comm, packed, M, s));
        DH_TRY(dh_loop_commit(B, L, k, steps, final_pass, packed, sel_rows, sel_count, tokens, active, need_eval,
                              counters, s));
    }
    return DH_OK;
}

}  // extern "C"
