// ref_shim.cpp -- plain C entry points over the reference's own HLS C++.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file together with
// the unmodified reference sources (hls/rng/philox_rng.cpp,
// hls/output_head/output_head.cpp, hls/candidate_sampler/candidate_sampler.cpp,
// hls/tensor_engine/int8_mac_tile.cpp, read in place from the reference tree)
// into oracle/_ref/libdh_ref.so.  The reference kernels take C++ stream
// objects; these wrappers convert them to flat arrays so ctypes can call them.
// Nothing here is shipped or used by the product path.
#include <cstdint>
#include <cstring>

#include "rng/philox_rng.hpp"
#include "output_head/output_head.hpp"
#include "candidate_sampler/candidate_sampler.hpp"

using namespace diffusion_accel;

extern "C" {

void ref_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
    PhiloxCounter c = {ctr[0], ctr[1], ctr[2], ctr[3]};
    PhiloxKey k = {key[0], key[1]};
    PhiloxCounter r = philox4x32_10(c, k);
    for (int i = 0; i < 4; ++i) out[i] = r[i];
}

int32_t ref_gumbel_q10(uint32_t word) { return factorized_gumbel_score_q10(word); }

uint32_t ref_gumbel_lut_address(uint32_t word) { return gumbel_lut_address(word); }

// Word / score streams in the reference order (vocab tile of 16, position,
// lane block of 4).  `out` must hold positions * vocabulary entries.
uint32_t ref_philox_word_stream(uint32_t* out, uint32_t positions, uint32_t vocabulary,
                                uint32_t evaluation_id, uint32_t stream_id,
                                uint32_t seed_low, uint32_t seed_high) {
    PhiloxWordStream s;
    uint32_t status = philox_word_stream_kernel(s, positions, vocabulary, evaluation_id,
                                                stream_id, seed_low, seed_high);
    if (status != kRngKernelOk) return status;
    size_t n = static_cast<size_t>(positions) * vocabulary;
    for (size_t i = 0; i < n; ++i) out[i] = s.read();
    return status;
}

uint32_t ref_philox_gumbel_stream(int32_t* out, uint32_t positions, uint32_t vocabulary,
                                  uint32_t evaluation_id, uint32_t stream_id,
                                  uint32_t seed_low, uint32_t seed_high) {
    GumbelScoreStream s;
    uint32_t status = philox_gumbel_stream_kernel(s, positions, vocabulary, evaluation_id,
                                                  stream_id, seed_low, seed_high);
    if (status != kRngKernelOk) return status;
    size_t n = static_cast<size_t>(positions) * vocabulary;
    for (size_t i = 0; i < n; ++i) out[i] = s.read();
    return status;
}

// output_head_int8_kernel with the noise given as a [positions, vocabulary]
// row-major array; it is fed to the kernel in the reference stream order.
uint32_t ref_output_head_int8(const int8_t* hidden, const int8_t* weights,
                              const int32_t* mult_q20, const int32_t* bias,
                              const int32_t* noise, uint16_t* candidates,
                              uint32_t positions, uint32_t hidden_size,
                              uint32_t vocabulary, uint32_t mask_token) {
    OutputHeadNoiseStream s;
    if (positions >= 1 && positions <= kOutputHeadMaxPositions) {
        for (uint32_t base = 0; base < vocabulary; base += kOutputHeadVocabularyTile)
            for (uint32_t p = 0; p < positions; ++p)
                for (uint32_t lane = 0; lane < kOutputHeadVocabularyTile; ++lane) {
                    uint32_t t = base + lane;
                    if (t < vocabulary) s.write(noise[static_cast<size_t>(p) * vocabulary + t]);
                }
    }
    uint16_t c[kOutputHeadMaxPositions] = {};
    uint32_t status = output_head_int8_kernel(hidden, weights, mult_q20, bias, s, c, positions,
                                              hidden_size, vocabulary, mask_token);
    if (status == kOutputHeadKernelOk) std::memcpy(candidates, c, positions * sizeof(uint16_t));
    return status;
}

// candidate_reveal_kernel on caller arrays sized for kCandidateMaxPositions.
uint64_t ref_candidate_reveal(uint16_t* tokens, const uint16_t* cands, uint64_t* active,
                              uint64_t* valid, const uint32_t* words, uint64_t threshold,
                              uint32_t positions) {
    return candidate_reveal_kernel(tokens, cands, active, valid, words, threshold, positions);
}

uint32_t ref_candidate_max_positions() { return kCandidateMaxPositions; }

}  // extern "C"
