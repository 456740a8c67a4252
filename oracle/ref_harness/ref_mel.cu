// Reference-kernel harness, log-mel frontend.  TEST INFRASTRUCTURE ONLY.
//
// Compiles the reference's own mel_frontend.cu (VideoLingo-user
// native/asr/src/mel_frontend.cu, included from where it lies; nothing is
// copied) and exposes its host entry point compute_mel_batched (:209-291),
// which allocates, uploads, runs its five kernels and copies back itself.
#include "mel_frontend.cu"

#include <cstring>

extern "C" int vlref_compute_mel_batched(const float* pcm, int chunks, float* out) {
  try {
    std::vector<float> in(pcm, pcm + static_cast<size_t>(chunks) * kChunkSamples);
    const MelOutput mel = compute_mel_batched(in, chunks);
    std::memcpy(out, mel.features.data(), mel.features.size() * sizeof(float));
    return 0;
  } catch (const std::exception&) {
    return 1;
  }
}
