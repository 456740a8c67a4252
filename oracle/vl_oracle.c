/*
 * vl_oracle.c - CPU restatement of the reference algorithms of the GLM-ASR
 * native layer ops.  TEST INFRASTRUCTURE ONLY: the parity tests, the smoke
 * check and the bench's CPU-baseline leg call it as the checker; the product
 * library (libvlasr.so) never links or calls it.
 *
 * Each function follows one reference kernel of VideoLingo-user
 * native/asr/src at its rounding points, in plain C (fp32 arithmetic with a
 * single rounding to the storage type, fp64 where the reference uses host
 * double tables).  Where the reference relies on nvcc contracting a*b+c into
 * one FMA, fmaf() is written out.  Storage types are passed as codes
 * (0 = f32, 1 = f16, 2 = bf16); arrays are float32 holding values that are
 * representable in the storage type, and every stored result is rounded to
 * it (round to nearest even).
 *
 * Summation orders mirror the reference's 256-thread blocks: thread t
 * accumulates elements t, t+256, ... and the partials are then added in
 * thread order (engine.cu:170-183, decoder.cu:89-97).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define OR_F32 0
#define OR_F16 1
#define OR_BF16 2

static float round_bf16(float x) {
  uint32_t u;
  memcpy(&u, &x, 4);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) {
    u |= 0x00400000u; /* quiet NaN */
  } else {
    u += 0x7fffu + ((u >> 16) & 1u);
  }
  u &= 0xffff0000u;
  memcpy(&x, &u, 4);
  return x;
}

static float round_f16(float x) { return (float)(_Float16)x; }

float or_round(int dtype, float x) {
  if (dtype == OR_BF16) return round_bf16(x);
  if (dtype == OR_F16) return round_f16(x);
  return x;
}

void or_round_array(int dtype, float* x, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = or_round(dtype, x[i]);
}

/* Block-of-256 strided sums: s = sum(v), q = sum(v*v) in the reference order. */
static void block_sums(const float* v, int64_t n, float* s, float* q) {
  float ps[256], pq[256];
  for (int t = 0; t < 256; ++t) {
    float a = 0.f, b = 0.f;
    for (int64_t i = t; i < n; i += 256) {
      a += v[i];
      b = fmaf(v[i], v[i], b); /* local_sq += v * v contracts to FFMA */
    }
    ps[t] = a;
    pq[t] = b;
  }
  float a = 0.f, b = 0.f;
  for (int t = 0; t < 256; ++t) {
    a += ps[t];
    b += pq[t];
  }
  *s = a;
  *q = b;
}

/*
 * Residual add + LayerNorm (engine.cu:207-212 then :162-192).
 * delta may be NULL (plain LN of residual, residual untouched).
 */
void or_add_layernorm(float* residual, const float* delta, const float* gamma, const float* beta,
                      float* out, int64_t rows, int64_t cols, float eps, int dtype) {
  float* h = (float*)malloc(sizeof(float) * (size_t)cols);
  for (int64_t r = 0; r < rows; ++r) {
    float* x = residual + r * cols;
    for (int64_t c = 0; c < cols; ++c) {
      h[c] = delta ? or_round(dtype, x[c] + delta[r * cols + c]) : x[c];
      if (delta) x[c] = h[c];
    }
    float s, q;
    block_sums(h, cols, &s, &q);
    const float mean = s / (float)cols;
    const float sq_mean = q / (float)cols;
    float var = fmaf(-mean, mean, sq_mean);
    if (var < 0.f) var = 0.f;
    const float inv = 1.0f / sqrtf(var + eps);
    for (int64_t c = 0; c < cols; ++c) {
      const float normalized = (h[c] - mean) * inv;
      const float b = beta ? beta[c] : 0.f;
      out[r * cols + c] = or_round(dtype, fmaf(normalized, gamma[c], b));
    }
  }
  free(h);
}

/* Residual add + RMSNorm (decoder.cu:933-938 then :81-101). */
void or_add_rmsnorm(float* residual, const float* delta, const float* weight, float* out,
                    int64_t rows, int64_t cols, float eps, int dtype) {
  float* h = (float*)malloc(sizeof(float) * (size_t)cols);
  for (int64_t r = 0; r < rows; ++r) {
    float* x = residual + r * cols;
    for (int64_t c = 0; c < cols; ++c) {
      h[c] = delta ? or_round(dtype, x[c] + delta[r * cols + c]) : x[c];
      if (delta) x[c] = h[c];
    }
    float s, q;
    block_sums(h, cols, &s, &q);
    const float inv = 1.0f / sqrtf(q / (float)cols + eps);
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = or_round(dtype, h[c] * inv * weight[c]);
  }
  free(h);
}

static float gelu_ref(float x) { return 0.5f * x * (1.0f + erff(x * 0.70710678118654752440f)); }

/* add_bias_kernel (engine.cu:200-205) then gelu_kernel (engine.cu:194-198). */
void or_gelu(const float* in, const float* bias, float* out, int64_t rows, int64_t cols,
             int dtype) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) {
      float x = in[r * cols + c];
      if (bias) x = or_round(dtype, x + bias[c]);
      out[r * cols + c] = or_round(dtype, gelu_ref(x));
    }
}

/* silu_mul_kernel (decoder.cu:103-109). */
void or_swiglu(const float* gate, const float* up, float* out, int64_t n, int dtype) {
  for (int64_t i = 0; i < n; ++i) {
    const float g = gate[i];
    out[i] = or_round(dtype, g / (1.0f + expf(-g)) * up[i]);
  }
}

/*
 * Rotate-half RoPE in place (engine.cu:214-233 with build_rope_table
 * :892-905; decoder.cu rope kernels with build_full_rope_table :950-961).
 * q [tokens][nq][head_dim], k [tokens][nk][head_dim] contiguous; positions
 * [tokens].
 */
void or_rope(float* q, float* k, const int64_t* positions, int64_t tokens, int nq, int nk,
             int head_dim, int rotary_dim, double base, int dtype) {
  const int half = rotary_dim / 2;
  for (int64_t t = 0; t < tokens; ++t) {
    for (int d = 0; d < half; ++d) {
      const double freq = 1.0 / pow(base, (double)(2 * d) / rotary_dim);
      const double angle = freq * (double)positions[t];
      const float c = (float)cos(angle), s = (float)sin(angle);
      for (int h = 0; h < nq + nk; ++h) {
        float* p = h < nq ? q + (t * nq + h) * (int64_t)head_dim
                          : k + (t * nk + (h - nq)) * (int64_t)head_dim;
        const float x1 = p[d], x2 = p[d + half];
        p[d] = or_round(dtype, fmaf(x1, c, -(x2 * s)));
        p[d + half] = or_round(dtype, fmaf(x2, c, x1 * s));
      }
    }
  }
}

/* ------------------------------------------------------------------------ */
/* Log-mel (mel_frontend.cu)                                                 */
/* ------------------------------------------------------------------------ */

#define MEL_BINS 128
#define N_FFT 400
#define N_FREQ 201
#define HOP 160
#define CHUNK 480000
#define FRAMES_ALL 3001
#define FRAMES 3000

static double hz_to_mel(double hz) {
  const double min_log_hz = 1000.0, min_log_mel = 15.0, logstep = 27.0 / log(6.4);
  if (hz < min_log_hz) return 3.0 * hz / 200.0;
  return min_log_mel + log(hz / min_log_hz) * logstep;
}

static double mel_to_hz(double mel) {
  const double min_log_hz = 1000.0, min_log_mel = 15.0, logstep = log(6.4) / 27.0;
  const double linear = 200.0 * mel / 3.0;
  if (mel < min_log_mel) return linear;
  return min_log_hz * exp(logstep * (mel - min_log_mel));
}

/* build_mel_filterbank (mel_frontend.cu:35-82): fb[k][m], k < 201, m < 128 (fp64). */
void or_mel_filterbank(double* fb) {
  double mel_points[MEL_BINS + 2], filter_freqs[MEL_BINS + 2], fft_freqs[N_FREQ];
  const double fmax = 8000.0;
  const double mel_min = hz_to_mel(0.0), mel_max = hz_to_mel(fmax);
  for (int i = 0; i < MEL_BINS + 2; ++i) {
    mel_points[i] = mel_min + (mel_max - mel_min) * i / (double)(MEL_BINS + 1);
    filter_freqs[i] = mel_to_hz(mel_points[i]);
  }
  for (int i = 0; i < N_FREQ; ++i) fft_freqs[i] = fmax * i / (double)(N_FREQ - 1);
  for (int m = 0; m < MEL_BINS; ++m) {
    const double left = filter_freqs[m], mid = filter_freqs[m + 1], right = filter_freqs[m + 2];
    const double enorm = 2.0 / (right - left);
    for (int k = 0; k < N_FREQ; ++k) {
      const double rising = (fft_freqs[k] - left) / (mid - left);
      const double falling = (right - fft_freqs[k]) / (right - mid);
      double v = rising < falling ? rising : falling;
      if (v < 0.0) v = 0.0;
      fb[k * MEL_BINS + m] = v * enorm;
    }
  }
}

static int reflect_index(int j, int n) {
  if (j < 0) return -j;
  if (j >= n) return 2 * n - 2 - j;
  return j;
}

/*
 * compute_mel_batched (mel_frontend.cu:209-291) as the reference computes it:
 * direct 400-tap DFT in fp32 with fp64-built windowed trig tables rounded to
 * f32 (stft_power_kernel :164-184), dense filterbank product
 * (mel_matmul_kernel :187-201), log10/max/normalise (:108-153).
 * pcm [chunks][480000] -> out [chunks][128][3000].
 */
void or_logmel_ref(const float* pcm, int64_t chunks, float* out) {
  double* fbd = (double*)malloc(sizeof(double) * N_FREQ * MEL_BINS);
  float* fb = (float*)malloc(sizeof(float) * N_FREQ * MEL_BINS);
  float* wcos = (float*)malloc(sizeof(float) * N_FREQ * N_FFT);
  float* wsin = (float*)malloc(sizeof(float) * N_FREQ * N_FFT);
  float* power = (float*)malloc(sizeof(float) * N_FREQ);
  float* frame = (float*)malloc(sizeof(float) * N_FFT);
  or_mel_filterbank(fbd);
  for (int i = 0; i < N_FREQ * MEL_BINS; ++i) fb[i] = (float)fbd[i];
  for (int k = 0; k < N_FREQ; ++k)
    for (int n = 0; n < N_FFT; ++n) {
      const double window = 0.5 * (1.0 - cos(2.0 * M_PI * n / N_FFT));
      const double angle = 2.0 * M_PI * ((double)k * n / N_FFT);
      wcos[k * N_FFT + n] = (float)(window * cos(angle));
      wsin[k * N_FFT + n] = (float)(window * sin(angle));
    }
  for (int64_t c = 0; c < chunks; ++c) {
    const float* x = pcm + c * CHUNK;
    float* o = out + c * (int64_t)MEL_BINS * FRAMES;
    float chunk_max = -1e30f;
    for (int f = 0; f < FRAMES; ++f) {
      const int start = f * HOP - N_FFT / 2;
      for (int n = 0; n < N_FFT; ++n) frame[n] = x[reflect_index(start + n, CHUNK)];
      for (int k = 0; k < N_FREQ; ++k) {
        float re = 0.f, im = 0.f;
        for (int n = 0; n < N_FFT; ++n) {
          re = fmaf(frame[n], wcos[k * N_FFT + n], re);
          im = fmaf(frame[n], wsin[k * N_FFT + n], im);
        }
        power[k] = fmaf(re, re, im * im);
      }
      for (int m = 0; m < MEL_BINS; ++m) {
        float sum = 0.f;
        for (int k = 0; k < N_FREQ; ++k) sum = fmaf(fb[k * MEL_BINS + m], power[k], sum);
        const float v = log10f(fmaxf(sum, 1e-10f));
        o[(int64_t)m * FRAMES + f] = v;
        if (v > chunk_max) chunk_max = v;
      }
    }
    const float floor_log = chunk_max - 8.0f;
    for (int64_t i = 0; i < (int64_t)MEL_BINS * FRAMES; ++i)
      o[i] = (fmaxf(o[i], floor_log) + 4.0f) / 4.0f;
  }
  free(fbd);
  free(fb);
  free(wcos);
  free(wsin);
  free(power);
  free(frame);
}

/* ------------------------------------------------------------------------ */
/* Decode step (decoder.cu:471-572, launched at :1710-1722)                  */
/* ------------------------------------------------------------------------ */

/*
 * rope_at_position_map_kernel + append_kv_mapped_kernel +
 * attention_step_mapped_kernel for `tokens` rows.  q [tokens][nq*hd],
 * k_new / v_new [tokens][nkv*hd] (NULL: the cache already holds position p),
 * caches [num_slots][nkv*hd].  Token t at position p = positions[t] uses
 * cache slots seq_start[t] + 0..p.  With rot > 0 q and k_new are rotated at
 * p (fp64 angle, fp32 cos/sin, results rounded to the storage type, as the
 * reference stores them), k_new / v_new are written to slot seq_start[t]+p.
 * Scores dot*scale (fp32, dims in order), softmax with max, expf and the sum
 * in position order, normalised probabilities, out = sum_t p_t v_t in
 * position order, rounded once.  q_new / k_new are modified (rotated).
 */
void or_decode_attention(float* q, float* k_new, const float* v_new, float* k_cache,
                         float* v_cache, const int32_t* positions, const int64_t* seq_start,
                         int64_t tokens, int nq, int nkv, int hd, int rot, double base,
                         float scale, int dtype, float* out) {
  const int group = nq / nkv;
  const int64_t row = (int64_t)nkv * hd;
  for (int64_t t = 0; t < tokens; ++t) {
    const int64_t p = positions[t];
    float* qt = q + t * (int64_t)nq * hd;
    if (k_new != NULL) {
      float* kt = k_new + t * row;
      if (rot > 0) {
        const int64_t pos64 = p;
        or_rope(qt, kt, &pos64, 1, nq, nkv, hd, rot, base, dtype);
      }
      memcpy(k_cache + (seq_start[t] + p) * row, kt, (size_t)row * sizeof(float));
      memcpy(v_cache + (seq_start[t] + p) * row, v_new + t * row, (size_t)row * sizeof(float));
    }
    float* scores = (float*)malloc((size_t)(p + 1) * sizeof(float));
    for (int h = 0; h < nq; ++h) {
      const int kvh = h / group;
      const float* qh = qt + (int64_t)h * hd;
      float mx = -INFINITY;
      for (int64_t s = 0; s <= p; ++s) {
        const float* kr = k_cache + (seq_start[t] + s) * row + (int64_t)kvh * hd;
        float dot = 0.0f;
        for (int d = 0; d < hd; ++d) dot = fmaf(qh[d], kr[d], dot);
        scores[s] = dot * scale;
        if (scores[s] > mx) mx = scores[s];
      }
      float total = 0.0f;
      for (int64_t s = 0; s <= p; ++s) {
        scores[s] = expf(scores[s] - mx);
        total += scores[s];
      }
      const float inv = 1.0f / total;
      for (int64_t s = 0; s <= p; ++s) scores[s] *= inv;
      for (int d = 0; d < hd; ++d) {
        float acc = 0.0f;
        for (int64_t s = 0; s <= p; ++s)
          acc = fmaf(scores[s], v_cache[(seq_start[t] + s) * row + (int64_t)kvh * hd + d], acc);
        out[(t * nq + h) * (int64_t)hd + d] = or_round(dtype, acc);
      }
    }
    free(scores);
  }
}

/*
 * Greedy next token with the EOS freeze: argmax_mapped_kernel
 * (decoder.cu:573-621); with finished == NULL, argmax_rows_kernel
 * (decoder.cu:755-782).  Logits are float32 holding storage values.
 *
 * Per row r (chunk c = row_chunk ? row_chunk[r] : r), as the reference's
 * 256-thread block computes it: thread t scans j = t, t+256, ... from -1e30
 * and keeps the first strictly greater value; thread 0 then scans the
 * threads in order from -1e30 and keeps the first strictly greater one.  A
 * row with no value above -1e30 yields freeze_id when finished is given
 * (the mapped kernel's initial winner) and 0 otherwise.
 * With finished: a finished chunk yields freeze_id and nothing else
 * changes; otherwise out_ids[(positions[c] - prompt_length + 1) *
 * out_stride + c] = id (when out_ids and the row is in [0, out_rows)) and
 * the chunk becomes finished when id is one of eos[0..n_eos).  current_ids[c]
 * = id in every case.
 */
void or_argmax_eos(const float* logits, int64_t rows, int64_t vocab, const int32_t* row_chunk,
                   uint8_t* finished, int64_t* current_ids, int64_t* out_ids,
                   const int32_t* positions, int64_t prompt_length, int64_t out_rows,
                   int64_t out_stride, const int64_t* eos, int n_eos, int64_t freeze_id) {
  enum { kThreads = 256 };
  for (int64_t r = 0; r < rows; ++r) {
    const int64_t c = row_chunk ? row_chunk[r] : r;
    if (finished && finished[c]) {
      current_ids[c] = freeze_id;
      continue;
    }
    const float* row = logits + r * vocab;
    float local_best[kThreads];
    int64_t local_index[kThreads];
    for (int t = 0; t < kThreads; ++t) {
      float best = -1e30f;
      int64_t index = 0;
      for (int64_t j = t; j < vocab; j += kThreads) {
        if (row[j] > best) {
          best = row[j];
          index = j;
        }
      }
      local_best[t] = best;
      local_index[t] = index;
    }
    float overall = -1e30f;
    int64_t winner = finished ? freeze_id : 0;
    for (int t = 0; t < kThreads; ++t) {
      if (local_best[t] > overall) {
        overall = local_best[t];
        winner = local_index[t];
      }
    }
    if (finished) {
      if (out_ids) {
        const int64_t orow = (int64_t)positions[c] - prompt_length + 1;
        if (orow >= 0 && orow < out_rows) out_ids[orow * out_stride + c] = winner;
      }
      for (int e = 0; e < n_eos; ++e)
        if (winner == eos[e]) finished[c] = 1;
    }
    current_ids[c] = winner;
  }
}
