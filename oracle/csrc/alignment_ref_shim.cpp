// C entry points over the reference's host alignment controller class
// (src/runtime/alignment_controller.hpp:43-66).  Compiled together with the
// reference's own src/runtime/alignment_controller.cpp, where it lies, into
// oracle/_ref/libalignment_ref.so by oracle/alignment_ref.py.  TEST
// INFRASTRUCTURE ONLY: it pins oracle/alignment.py and produces the golden
// vectors under tests/golden/; the product library never links it.
#include <cstdint>
#include <cstring>
#include <new>
#include <vector>

#include "runtime/alignment_controller.hpp"

namespace {

using magpie_tts_rt::AlignmentControllerError;
using magpie_tts_rt::AlignmentControllerErrorCode;
using magpie_tts_rt::AlignmentControllerReference;
using magpie_tts_rt::AlignmentManifest;

// 0 = ok, 1 + the error code's position in alignment_controller.hpp:12-17,
// 99 = any other exception.
int status_of(const AlignmentControllerError& e) {
  switch (e.code()) {
    case AlignmentControllerErrorCode::invalid_text_length: return 1;
    case AlignmentControllerErrorCode::invalid_score_count: return 2;
    case AlignmentControllerErrorCode::non_finite_score: return 3;
    case AlignmentControllerErrorCode::state_overflow: return 4;
  }
  return 99;
}

}  // namespace

extern "C" {

void* mtt_ref_alignment_create(uint32_t text_length, double prior_epsilon, uint32_t initial_attended,
                               uint32_t ignored_terminal_tokens, uint32_t short_text_no_prior_max_tokens,
                               uint32_t lookahead, uint32_t sink_threshold, int* status) {
  AlignmentManifest m{};
  m.prior_epsilon = prior_epsilon;
  m.initial_attended = initial_attended;
  m.ignored_terminal_tokens = ignored_terminal_tokens;
  m.short_text_no_prior_max_tokens = short_text_no_prior_max_tokens;
  m.lookahead = lookahead;
  m.sink_threshold = sink_threshold;
  try {
    auto* c = new AlignmentControllerReference(text_length, m);
    *status = 0;
    return c;
  } catch (const AlignmentControllerError& e) {
    *status = status_of(e);
  } catch (...) {
    *status = 99;
  }
  return nullptr;
}

int mtt_ref_alignment_advance(void* handle, const float* scores, uint32_t count, uint32_t* attended,
                              int32_t* unfinished, float* next_prior, uint32_t prior_capacity) {
  auto* c = static_cast<AlignmentControllerReference*>(handle);
  try {
    const auto r = c->advance(std::vector<float>(scores, scores + count));
    *attended = r.attended_token_index;
    *unfinished = r.unfinished_text ? 1 : 0;
    if (r.next_prior.size() > prior_capacity) return 98;
    std::memcpy(next_prior, r.next_prior.data(), r.next_prior.size() * sizeof(float));
    return 0;
  } catch (const AlignmentControllerError& e) {
    return status_of(e);
  } catch (...) {
    return 99;
  }
}

uint32_t mtt_ref_alignment_last_attended(void* handle) {
  return static_cast<AlignmentControllerReference*>(handle)->last_attended_token_index();
}

void mtt_ref_alignment_counters(void* handle, uint32_t* out) {
  const auto& v = static_cast<AlignmentControllerReference*>(handle)->counters();
  std::memcpy(out, v.data(), v.size() * sizeof(uint32_t));
}

void mtt_ref_alignment_destroy(void* handle) { delete static_cast<AlignmentControllerReference*>(handle); }

}  // extern "C"
