// Reference-engine harness, audio tower + projector.  TEST INFRASTRUCTURE ONLY.
//
// Drives the reference's own public engine API (VideoLingo-user
// native/asr/src/engine.h:20-76 and model_loader.h; compiled from its sources
// where they lie, nothing copied): load_weights_resident reads a checkpoint
// directory (config.json + BF16 model.safetensors with the official
// inventory) into FP16 device weights, and run_encode_batched runs mel
// [chunks,128,3000] through conv frontend, 32 encoder layers, final norm and
// projector into a caller-allocated FP16 [chunks*375, 2048] device buffer.
// C++ exceptions are caught here and turned into status codes (2 = the
// reference's ModelInputError, 1 = anything else) with the message kept for
// vlref_last_error().
#include <exception>
#include <string>
#include <vector>

#include "engine.h"
#include "model_loader.h"

namespace {
thread_local std::string g_error;

int fail(const std::exception& e, int code) {
  g_error = e.what();
  return code;
}
}  // namespace

extern "C" {

const char* vlref_last_error() { return g_error.c_str(); }

// Returns an owned DeviceWeights* or nullptr (message in vlref_last_error).
void* vlref_load_weights(const char* model_dir, unsigned long long max_vram_bytes) {
  try {
    return new DeviceWeights(load_weights_resident(model_dir, max_vram_bytes));
  } catch (const std::exception& e) {
    fail(e, 1);
    return nullptr;
  }
}

void vlref_free_weights(void* weights) { delete static_cast<DeviceWeights*>(weights); }

unsigned long long vlref_weights_bytes(void* weights) {
  return static_cast<DeviceWeights*>(weights)->device_bytes();
}

// mel: host f32 [chunks,128,3000]; projector_out: device FP16 [chunks*375,2048].
int vlref_encode_batched(void* weights, const float* mel, int chunks, int fp16_accumulate,
                         void* projector_out) {
  try {
    const size_t count = static_cast<size_t>(chunks > 0 ? chunks : 0) * 128 * 3000;
    std::vector<float> features(mel, mel + count);
    EncodeOptions options;
    options.fp16_accumulate = fp16_accumulate != 0;
    options.dump_stages = false;
    run_encode_batched(features, chunks, static_cast<DeviceWeights*>(weights), options,
                       static_cast<uint16_t*>(projector_out));
    return 0;
  } catch (const ModelInputError& e) {
    return fail(e, 2);
  } catch (const std::exception& e) {
    return fail(e, 1);
  }
}

// Cross-chunk batched decode (engine.h:95-105, decoder.cu:1372-1800):
// audio_embeds is the device FP16 projector output [chunks*375, 2048];
// prompt_ids (host) are shared by every chunk.  out_ids (host) receives
// [chunks][max_new_tokens] ids, -1 after each chunk's last id (its EOS or
// the budget); out_lens the count per chunk; the engine's own prefill and
// decode times are returned in milliseconds.
int vlref_decode_batched(void* weights, const void* audio_embeds, int chunks,
                         const int64_t* prompt_ids, int prompt_len, int max_new_tokens,
                         int fp16_accumulate, int64_t* out_ids, int* out_lens, float* prefill_ms,
                         float* decode_ms) {
  try {
    std::vector<int64_t> prompt(prompt_ids, prompt_ids + (prompt_len > 0 ? prompt_len : 0));
    DecodeOptions options;
    options.fp16_accumulate = fp16_accumulate != 0;
    options.max_new_tokens = max_new_tokens;
    options.prefill_batched = true;
    const DecodeBatchResult r =
        run_decode_batched(static_cast<DeviceWeights*>(weights),
                           static_cast<const uint16_t*>(audio_embeds), chunks, prompt, options);
    for (int c = 0; c < chunks; ++c) {
      const std::vector<int64_t>& ids = r.per_chunk_ids[static_cast<size_t>(c)];
      int n = 0;
      for (; n < max_new_tokens && n < static_cast<int>(ids.size()); ++n)
        out_ids[static_cast<size_t>(c) * max_new_tokens + n] = ids[static_cast<size_t>(n)];
      out_lens[c] = n;
      for (int i = n; i < max_new_tokens; ++i)
        out_ids[static_cast<size_t>(c) * max_new_tokens + i] = -1;
    }
    if (prefill_ms) *prefill_ms = r.prefill_ms;
    if (decode_ms) *decode_ms = r.decode_ms;
    return 0;
  } catch (const ModelInputError& e) {
    return fail(e, 2);
  } catch (const std::exception& e) {
    return fail(e, 1);
  }
}

}  // extern "C"
