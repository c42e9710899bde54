// stream.cu -- streaming transcription (crates/qwen-asr/src/transcribe.rs):
// transcribe_stream (445-800) and the incremental stream_push_audio with its
// StreamState (809-1495), on the device engines, token ids out.
//
// Per chunk of chunk_sec audio: the encoder output of every completed 8 s
// window is computed once and cached on the device; the partial tail window
// is re-encoded (in incremental mode only every second chunk, reusing the
// previous tail otherwise); the prompt rows (special tokens, cached windows,
// tail, suffix, forced tokens and, with past-text conditioning, the committed
// tokens minus the rollback) are assembled on the device; the longest common
// prefix with the previous chunk's prompt rows is found on the device and
// only the rows after it are prefilled into the KV cache (the rows before it
// are still there); then a greedy decode of up to max_new_tokens.  The host
// keeps the token bookkeeping of the reference: degeneracy resets (a stale
// or periodically repeating tail), re-anchoring (every 45 chunks or at 200
// encoder rows), the rollback frontier, the monotonic commit of stable
// tokens and, incrementally, the byte-level realignment after a re-anchor
// (token byte lengths supplied by the caller, who holds the tokenizer).
//
// The stream decodes in KV slot 0 of its decoder (batch of one).
#include <algorithm>
#include <cstring>
#include <deque>
#include <vector>

#include "common.cuh"
#include "engine.cuh"
#include "matvec.cuh"

namespace qasr {
namespace {

constexpr int kDegenMaxPeriod = 6, kDegenMinRepeats = 4, kStaleChunks = 4, kResetInterval = 45, kCarryTokens = 24;
constexpr int kReanchorEncRows = 200;  // transcribe.rs:16-27
constexpr int kDecodeCheck = 8;

// *first = the first row in [0, rows) where a and b differ (f32 !=), else rows.
__global__ void __launch_bounds__(256) first_diff_row_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                                             int rows, int cols, int *__restrict__ first) {
  const int lane = threadIdx.x & 31;
  for (int r = blockIdx.x * 8 + (threadIdx.x >> 5); r < rows; r += gridDim.x * 8) {
    // an earlier row already differs: lane 0's read decides for the whole warp
    const int known = __shfl_sync(0xffffffffu, *reinterpret_cast<volatile int *>(first), 0);
    if (r >= known) break;
    bool diff = false;
    for (int c = lane; c < cols; c += 32) diff |= a[(size_t)r * cols + c] != b[(size_t)r * cols + c];
    if (__any_sync(0xffffffffu, diff) && lane == 0) atomicMin(first, r);
  }
}

struct EncWin {
  float *rows = nullptr;
  int seq = 0;
};

}  // namespace

// stream_tail_repeat_blocks (transcribe.rs:42-59): the largest number of
// times a block of p <= max_period tokens repeats at the tail, and that p.
void tail_repeat_blocks(const int32_t *t, int n, int max_period, int *best_reps, int *best_period) {
  *best_reps = 1;
  *best_period = 0;
  if (n < 2) return;
  const int cap = std::min(n / 2, max_period > 0 ? max_period : n / 2);
  for (int p = 1; p <= cap; ++p) {
    int reps = 1;
    while ((reps + 1) * p <= n && std::equal(t + n - (reps + 1) * p, t + n - reps * p, t + n - reps * p)) ++reps;
    if (reps > *best_reps) {
      *best_reps = reps;
      *best_period = p;
    }
  }
}

}  // namespace qasr

using namespace qasr;

struct qasr_stream {
  qasr_decoder *dec = nullptr;
  qasr_encoder *enc = nullptr;
  int device = 0, H = 0;
  cudaStream_t st = nullptr;
  qasr_stream_config cfg{};
  long chunk = 0, window = 0;
  std::vector<int32_t> prompt, force, tok_bytes;
  // encoder: completed windows (device rows), the tail window's latest encoding
  std::deque<EncWin> cache;
  long cached_rows = 0, base_windows = 0;
  float *tail = nullptr;
  int tail_cap = 0, tail_seq = 0;
  long tail_cursor = 0;
  // prompt rows of this chunk and of the previous one (device), LCP result
  float *rows = nullptr, *prev = nullptr;
  int rows_cap = 0, prev_cap = 0, prev_len = 0;
  int *d_first = nullptr;
  // token bookkeeping (StreamState)
  std::vector<int32_t> raw, stable, snapshot, emitted;
  int stale = 0, chunk_idx = 0;
  long cursor = 0, trim_request = 0;
};

namespace {

void free_window(EncWin &w) {
  if (w.rows) cudaFree(w.rows);
  w.rows = nullptr;
}

int grow(float **buf, int *cap, int rows, int H, const char *what) {
  if (rows <= *cap) return QASR_OK;
  if (*buf) cudaFree(*buf);
  *buf = nullptr;
  *cap = 0;
  int rc = cuda_status(cudaMalloc(buf, (size_t)std::max(rows, 64) * H * 4), what);
  if (!rc) *cap = std::max(rows, 64);
  return rc;
}

// keep the newest `keep` cached windows
void drop_windows(qasr_stream *s, int keep) {
  while ((int)s->cache.size() > keep) {
    s->cached_rows -= s->cache.front().seq;
    free_window(s->cache.front());
    s->cache.pop_front();
    ++s->base_windows;
  }
  s->cached_rows = std::max(0l, s->cached_rows);
}

int token_bytes(const qasr_stream *s, int32_t t) {
  return (t >= 0 && t < (int)s->tok_bytes.size()) ? s->tok_bytes[t] : 1;
}

}  // namespace

extern "C" int qasr_stream_tail_repeat(const int32_t *tokens, int n, int max_period, int *best_reps,
                                       int *best_period) {
  if ((n > 0 && !tokens) || !best_reps || !best_period) {
    set_error("qasr_stream_tail_repeat: invalid arguments");
    return QASR_ERR_INVALID;
  }
  tail_repeat_blocks(tokens, std::max(n, 0), max_period, best_reps, best_period);
  return QASR_OK;
}

// find_split_point (transcribe.rs:250-275): centre of the quietest 100 ms
// window (hop 50 ms) within +-search_sec of target_sample.
extern "C" int64_t qasr_find_split_point(const float *samples, int64_t n, int64_t target_sample, float search_sec) {
  if (!samples || n <= 0) return target_sample;
  const int64_t half = (int64_t)(search_sec * 16000.0f);
  const int64_t lo = target_sample > half ? target_sample - half : 0;
  const int64_t hi = std::min(target_sample + half, n);
  const int64_t win = 1600;
  float best = 1e30f;
  int64_t best_center = target_sample;
  for (int64_t pos = lo; pos + win <= hi; pos += win / 2) {
    const int64_t end = std::min(pos + win, n);
    float e = 0.0f;
    for (int64_t j = pos; j < end; ++j) e += samples[j] * samples[j];
    e /= (float)(end - pos);
    if (e < best) {
      best = e;
      best_center = pos + (end - pos) / 2;
    }
  }
  return best_center;
}

extern "C" void qasr_stream_default_config(qasr_stream_config *cfg) {
  if (!cfg) return;
  // QwenCtx defaults (context.rs:499-512): 2 s chunks, rollback 5, 2 unfixed
  // chunks, 32 new tokens, no past-text conditioning; StreamState semantics.
  cfg->chunk_sec = 2.0f;
  cfg->rollback = 5;
  cfg->unfixed_chunks = 2;
  cfg->max_new_tokens = 32;
  cfg->past_text_conditioning = 0;
  cfg->incremental = 1;
}

extern "C" void qasr_stream_free(qasr_stream *s) {
  if (!s) return;
  cudaSetDevice(s->device);
  if (s->st) cudaStreamSynchronize(s->st);
  for (EncWin &w : s->cache) free_window(w);
  if (s->tail) cudaFree(s->tail);
  if (s->rows) cudaFree(s->rows);
  if (s->prev) cudaFree(s->prev);
  if (s->d_first) cudaFree(s->d_first);
  delete s;
}

extern "C" qasr_stream *qasr_stream_create(qasr_decoder *dec, qasr_encoder *enc, const qasr_stream_config *cfg) {
  const qasr_decoder_config *dc = qasr_decoder_get_config(dec);
  const qasr_encoder_config *ec = qasr_encoder_get_config(enc);
  if (!dc || !ec || !cfg || cfg->chunk_sec <= 0.0f || cfg->rollback < 0 || cfg->unfixed_chunks < 0) {
    set_error("qasr_stream_create: invalid arguments");
    return nullptr;
  }
  if (ec->output_dim != dc->hidden || qasr_encoder_device(enc) != qasr_decoder_device(dec)) {
    set_error("qasr_stream_create: encoder and decoder do not match (output size or device)");
    return nullptr;
  }
  qasr_stream *s = new qasr_stream();
  s->dec = dec;
  s->enc = enc;
  s->device = qasr_decoder_device(dec);
  s->H = dc->hidden;
  s->st = reinterpret_cast<cudaStream_t>(qasr_decoder_stream(dec));
  s->cfg = *cfg;
  if (s->cfg.max_new_tokens <= 0) s->cfg.max_new_tokens = 32;
  s->chunk = (long)(cfg->chunk_sec * 16000.0f);
  s->window = (long)std::min(800, std::max(100, ec->n_window_infer)) * 160;  // enc_n_window_infer.clamp(100, 800) frames
  if (s->chunk <= 0 || cudaSetDevice(s->device) != cudaSuccess ||
      cudaMalloc(&s->d_first, sizeof(int)) != cudaSuccess) {
    set_error("qasr_stream_create: setup failed");
    qasr_stream_free(s);
    return nullptr;
  }
  return s;
}

// QwenCtx::prompt_tokens / force_prompt_tokens (ids of the caller's text prompt
// and forced language), placed as in transcribe_segment.
extern "C" int qasr_stream_set_prompt(qasr_stream *s, const int32_t *prompt, int n_prompt, const int32_t *force,
                                      int n_force) {
  if (!s || n_prompt < 0 || n_force < 0 || (n_prompt && !prompt) || (n_force && !force)) {
    set_error("qasr_stream_set_prompt: invalid arguments");
    return QASR_ERR_INVALID;
  }
  s->prompt.assign(prompt, prompt + n_prompt);
  s->force.assign(force, force + n_force);
  s->raw.clear();  // a new prompt invalidates the reusable prefix
  s->prev_len = 0;
  return QASR_OK;
}

// tokenizer.decode_bytes(t).len() for every id (the byte-level realignment of
// stream_push_audio); ids outside the table count one byte.
extern "C" int qasr_stream_set_token_bytes(qasr_stream *s, const int32_t *bytes, int n) {
  if (!s || n < 0 || (n && !bytes)) {
    set_error("qasr_stream_set_token_bytes: invalid arguments");
    return QASR_ERR_INVALID;
  }
  s->tok_bytes.assign(bytes, bytes + n);
  return QASR_OK;
}

// StreamState::reset (transcribe.rs:884-904): keeps the prompt and token bytes.
extern "C" int qasr_stream_reset(qasr_stream *s) {
  if (!s) return QASR_ERR_INVALID;
  cudaSetDevice(s->device);
  for (EncWin &w : s->cache) free_window(w);
  s->cache.clear();
  s->cached_rows = s->base_windows = 0;
  s->tail_seq = 0;
  s->tail_cursor = 0;
  s->prev_len = 0;
  s->raw.clear();
  s->stable.clear();
  s->snapshot.clear();
  s->emitted.clear();
  s->stale = s->chunk_idx = 0;
  s->cursor = s->trim_request = 0;
  return QASR_OK;
}

extern "C" int64_t qasr_stream_audio_cursor(const qasr_stream *s) { return s ? s->cursor : 0; }
extern "C" int64_t qasr_stream_trim_request(const qasr_stream *s) { return s ? s->trim_request : 0; }

// StreamState::apply_audio_trim (transcribe.rs:916-927): the caller dropped
// `trim` samples from the front of its buffer.
extern "C" int qasr_stream_apply_trim(qasr_stream *s, int64_t trim) {
  if (!s || trim < 0) return QASR_ERR_INVALID;
  s->cursor = std::max<int64_t>(0, s->cursor - trim);
  s->tail_cursor = std::max<int64_t>(0, s->tail_cursor - trim);
  s->base_windows = std::max<int64_t>(0, s->base_windows - trim / s->window);
  s->trim_request = 0;
  return QASR_OK;
}

// Every token committed so far (StreamState::text as ids), and the
// committed-but-rollback-pending tail (unfixed_text as ids).
extern "C" int qasr_stream_emitted(const qasr_stream *s, int32_t *ids, int cap, int *n) {
  if (!s || !n || (cap > 0 && !ids)) return QASR_ERR_INVALID;
  *n = (int)s->emitted.size();
  std::memcpy(ids, s->emitted.data(), (size_t)std::min(cap, *n) * 4);
  return QASR_OK;
}

extern "C" int qasr_stream_unfixed(const qasr_stream *s, int32_t *ids, int cap, int *n) {
  if (!s || !n || (cap > 0 && !ids)) return QASR_ERR_INVALID;
  const auto it = std::find(s->raw.begin(), s->raw.end(), kTokAsrText);
  const size_t text_start = it == s->raw.end() ? 0 : (size_t)(it - s->raw.begin()) + 1;
  const size_t n_text = s->raw.size() - text_start;
  *n = n_text > s->stable.size() ? (int)(n_text - s->stable.size()) : 0;
  std::memcpy(ids, s->raw.data() + text_start + s->stable.size(), (size_t)std::min(cap, *n) * 4);
  return QASR_OK;
}

namespace {

// Reference token bookkeeping after a chunk's decode, shared by the degeneracy
// reset and the re-anchor (transcribe.rs:677-755 / 1222-1346): carry the last
// committed tokens (behind an <asr_text> marker) and forget the prompt rows.
void carry_reset(qasr_stream *s, int keep_windows) {
  const size_t carry = std::min(s->stable.size(), (size_t)kCarryTokens);
  const std::vector<int32_t> carried(s->stable.end() - carry, s->stable.end());
  s->raw.clear();
  if (carry) {
    s->raw.push_back(kTokAsrText);
    s->raw.insert(s->raw.end(), carried.begin(), carried.end());
  }
  s->stable = carried;
  s->prev_len = 0;
  s->stale = 0;
  s->snapshot.clear();
  drop_windows(s, keep_windows);
  if (s->cfg.incremental && s->cursor > s->chunk * 4) s->trim_request = s->cursor - s->chunk * 4;
}

// One chunk: returns QASR_OK with *skipped set when there is no encoder output yet.
int stream_chunk(qasr_stream *s, const float *samples, long n, bool is_final, std::vector<int32_t> &delta,
                 bool *skipped) {
  const int H = s->H;
  const qasr_decoder_config *dc = qasr_decoder_get_config(s->dec);
  *skipped = false;
  int rc = QASR_OK;
  // ---- encoder: new completed windows, then the tail
  const long full_end = (s->cursor / s->window) * s->window;
  while ((s->base_windows + (long)s->cache.size()) * s->window < full_end) {
    const long ws = (s->base_windows + (long)s->cache.size()) * s->window;
    const int cap = qasr_encoder_tokens(s->enc, qasr_mel_frames((int)s->window));
    EncWin w;
    if ((rc = cuda_status(cudaMalloc(&w.rows, (size_t)cap * H * 4), "stream: window rows"))) return rc;
    if ((rc = encode_samples(s->enc, s->device, s->st, samples + ws, (int)s->window, w.rows, cap, &w.seq))) {
      free_window(w);
      return rc;
    }
    s->cached_rows += w.seq;
    s->cache.push_back(w);
  }
  int tail_seq = 0;
  if (full_end < s->cursor) {
    const long tail_n = s->cursor - full_end;
    const bool need = !s->cfg.incremental || s->tail_cursor == 0 || s->cursor - s->tail_cursor >= 2 * s->chunk ||
                      is_final;
    if (need && qasr_mel_frames((int)tail_n) > 0) {
      const int cap = qasr_encoder_tokens(s->enc, qasr_mel_frames((int)tail_n));
      if ((rc = grow(&s->tail, &s->tail_cap, cap, H, "stream: tail rows"))) return rc;
      if ((rc = encode_samples(s->enc, s->device, s->st, samples + full_end, (int)tail_n, s->tail, s->tail_cap,
                               &s->tail_seq)))
        return rc;
      s->tail_cursor = s->cursor;
      tail_seq = s->tail_seq;
    } else if (s->cfg.incremental) {
      tail_seq = s->tail_seq;  // the previous chunk's tail encoding, as stream_push_audio reuses it
    }
  }
  const long enc_rows = s->cached_rows + tail_seq;
  if (enc_rows == 0) {
    ++s->chunk_idx;
    *skipped = true;
    return QASR_OK;
  }
  // ---- prompt rows
  const int n_prefix = (s->cfg.past_text_conditioning && s->chunk_idx >= s->cfg.unfixed_chunks && !s->raw.empty())
                           ? std::max(0, (int)s->raw.size() - s->cfg.rollback)
                           : 0;
  std::vector<int32_t> pre(kPrefixHead, kPrefixHead + 3);
  pre.insert(pre.end(), s->prompt.begin(), s->prompt.end());
  pre.insert(pre.end(), kPrefixTail, kPrefixTail + 6);
  std::vector<int32_t> post(kSuffixBase, kSuffixBase + 6);
  post.insert(post.end(), s->force.begin(), s->force.end());
  post.insert(post.end(), s->raw.begin(), s->raw.begin() + n_prefix);
  const int total = (int)(pre.size() + enc_rows + post.size()), prefill_len = total - 1;
  if (prefill_len + s->cfg.max_new_tokens > dc->max_seq) {
    set_error("stream: %d prompt rows + %d new tokens exceed the cache (%d)", total, s->cfg.max_new_tokens,
              dc->max_seq);
    return QASR_ERR_INVALID;
  }
  if ((rc = grow(&s->rows, &s->rows_cap, total, H, "stream: prompt rows"))) return rc;
  if ((rc = qasr_decoder_embed(s->dec, pre.data(), (int)pre.size(), s->rows))) return rc;
  size_t r = pre.size();
  for (const EncWin &w : s->cache) {
    if ((rc = cuda_status(cudaMemcpyAsync(s->rows + r * H, w.rows, (size_t)w.seq * H * 4, cudaMemcpyDeviceToDevice,
                                          s->st),
                          "stream: window rows")))
      return rc;
    r += w.seq;
  }
  if (tail_seq &&
      (rc = cuda_status(cudaMemcpyAsync(s->rows + r * H, s->tail, (size_t)tail_seq * H * 4, cudaMemcpyDeviceToDevice,
                                        s->st),
                        "stream: tail rows")))
    return rc;
  r += tail_seq;
  if ((rc = qasr_decoder_embed(s->dec, post.data(), (int)post.size(), s->rows + r * H))) return rc;
  // ---- longest common prefix with the previous chunk's rows, prefill the rest
  int reused = 0;
  const int cmp = std::min(prefill_len, s->prev_len);
  if (cmp > 0) {
    if ((rc = cuda_status(cudaMemcpyAsync(s->d_first, &cmp, sizeof(int), cudaMemcpyHostToDevice, s->st), "stream: lcp")))
      return rc;
    first_diff_row_kernel<<<std::min((cmp + 7) / 8, 148 * 4), 256, 0, s->st>>>(s->prev, s->rows, cmp, H,
                                                                               s->d_first);
    if ((rc = launch_status("stream: lcp"))) return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(&reused, s->d_first, sizeof(int), cudaMemcpyDeviceToHost, s->st),
                          "stream: lcp")))
      return rc;
    if ((rc = cuda_status(cudaStreamSynchronize(s->st), "stream: lcp"))) return rc;
  }
  if (prefill_len > reused && (rc = qasr_decoder_prefill(s->dec, 0, s->rows + (size_t)reused * H,
                                                         prefill_len - reused, reused)))
    return rc;
  if ((rc = grow(&s->prev, &s->prev_cap, prefill_len, H, "stream: previous rows"))) return rc;
  if ((rc = cuda_status(cudaMemcpyAsync(s->prev, s->rows, (size_t)prefill_len * H * 4, cudaMemcpyDeviceToDevice,
                                        s->st),
                        "stream: previous rows")))
    return rc;
  s->prev_len = prefill_len;
  // ---- greedy decode from the last prompt token (stop tokens end it, not kept)
  const int32_t tok0 = post.back();
  const int32_t pos0 = prefill_len;
  std::vector<int32_t> ids(s->cfg.max_new_tokens);
  int n_ids = 0;
  if ((rc = greedy_decode(s->dec, 1, &tok0, &pos0, s->cfg.max_new_tokens, 1, kDecodeCheck, ids.data(),
                          s->cfg.max_new_tokens, &n_ids)))
    return rc;
  if (n_ids > 0 && is_stop_token(ids[n_ids - 1])) --n_ids;
  s->raw.resize(n_prefix);
  s->raw.insert(s->raw.end(), ids.begin(), ids.begin() + n_ids);
  // ---- degeneracy and re-anchoring
  if (s->raw == s->snapshot) {
    ++s->stale;
  } else {
    s->stale = 0;
    s->snapshot = s->raw;
  }
  int reps = 1, period = 0;
  tail_repeat_blocks(s->raw.data(), (int)s->raw.size(), kDegenMaxPeriod, &reps, &period);
  if (s->stale >= kStaleChunks || reps >= kDegenMinRepeats) carry_reset(s, s->cfg.incremental ? 1 : 2);
  if ((s->chunk_idx > 0 && s->chunk_idx % kResetInterval == 0) || enc_rows >= kReanchorEncRows) carry_reset(s, 1);
  // ---- commit: rollback frontier, byte realignment (incremental), emit
  const auto mark = std::find(s->raw.begin(), s->raw.end(), kTokAsrText);
  const size_t text_start = mark == s->raw.end() ? 0 : (size_t)(mark - s->raw.begin()) + 1;
  const std::vector<int32_t> cand(s->raw.begin() + text_start, s->raw.end());
  const size_t n_text = cand.size();
  size_t cand_len = 0;
  if (is_final)
    cand_len = n_text;
  else if (s->chunk_idx >= s->cfg.unfixed_chunks)
    cand_len = (size_t)std::max(0, (int)n_text - s->cfg.rollback);
  size_t emit_from = s->stable.size(), emit_to = std::max(cand_len, emit_from);
  if (s->cfg.incremental && emit_from > 0) {
    long mm = -1;
    for (size_t j = 0; j < std::min(emit_from, cand.size()); ++j)
      if (j < s->stable.size() && s->stable[j] != cand[j]) {
        mm = (long)j;
        break;
      }
    if (mm < 0 && s->stable.size() > cand.size()) mm = (long)cand.size();
    if (mm >= 0) {
      long stable_bytes = 0;
      for (long j = 0; j < mm; ++j) stable_bytes += token_bytes(s, s->stable[j]);
      size_t aligned = cand.size();
      long cum = 0;
      for (size_t j = 0; j < cand.size(); ++j) {
        cum += token_bytes(s, cand[j]);
        if (cum >= stable_bytes) {
          aligned = j + 1;
          break;
        }
      }
      aligned = std::min(aligned, cand.size());
      s->stable.assign(cand.begin(), cand.begin() + aligned);
      emit_from = aligned;
      emit_to = std::max(cand_len, emit_from);
    }
  }
  for (size_t i = emit_from; i < emit_to; ++i)
    if (i < cand.size()) {
      if (i >= s->stable.size()) s->stable.push_back(cand[i]);
      delta.push_back(cand[i]);
      s->emitted.push_back(cand[i]);
    }
  ++s->chunk_idx;
  return QASR_OK;
}

}  // namespace

// stream_push_audio (transcribe.rs:960-1495) with cfg.incremental set, else
// transcribe_stream (445-800) when given the whole buffer with finalize = 1.
// samples: everything received so far (host or device); emitted (host, cap
// entries) receives the ids committed by this call, *n_emitted their count.
extern "C" int qasr_stream_push(qasr_stream *s, const float *samples, int64_t n_samples, int finalize, int32_t *emitted,
                                int cap, int *n_emitted) {
  if (!s || (n_samples > 0 && !samples) || n_samples < 0 || !n_emitted || (cap > 0 && !emitted)) {
    set_error("qasr_stream_push: invalid arguments");
    return QASR_ERR_INVALID;
  }
  *n_emitted = 0;
  if (cudaSetDevice(s->device) != cudaSuccess) return QASR_ERR_CUDA;
  ArenaScope arena_scope(decoder_arena(s->dec));
  std::vector<int32_t> delta;
  int rc = QASR_OK;
  const long avail = n_samples > s->cursor ? n_samples - s->cursor : 0;
  if (s->cfg.incremental && ((avail < s->chunk && !finalize) || avail == 0)) return QASR_OK;
  while (s->cursor < n_samples) {
    if (s->cfg.incremental && n_samples - s->cursor < s->chunk && !finalize) break;
    s->cursor = std::min<long>(s->cursor + s->chunk, n_samples);
    const bool is_final = s->cfg.incremental ? (finalize && s->cursor >= n_samples) : s->cursor >= n_samples;
    bool skipped = false;
    if ((rc = stream_chunk(s, samples, n_samples, is_final, delta, &skipped))) return rc;
    if (skipped && s->cfg.incremental) {
      delta.clear();  // stream_push_audio returns an empty delta here
      break;
    }
  }
  *n_emitted = (int)delta.size();
  if ((int)delta.size() > cap) {
    set_error("qasr_stream_push: %d ids emitted, room for %d", (int)delta.size(), cap);
    return QASR_ERR_INVALID;
  }
  if (!delta.empty()) std::memcpy(emitted, delta.data(), delta.size() * 4);
  return QASR_OK;
}

// The segment plan of transcribe_audio (transcribe.rs:317-345): with
// segment_sec > 0 and more than segment_sec + the search margin of audio,
// split points every ~segment_sec at the quietest 100 ms within +-search of
// the target (search = min(search_sec, segment_sec / 2)), at most 127
// points.  starts[i] is the first sample of segment i (segment i ends at
// starts[i+1], the last at n); *n_segments their count (starts holds cap).
extern "C" int qasr_plan_segments(const float *samples, int64_t n, float segment_sec, float search_sec,
                                  int64_t *starts, int cap, int *n_segments) {
  if ((n > 0 && !samples) || n < 0 || !n_segments || (cap > 0 && !starts)) {
    set_error("qasr_plan_segments: invalid arguments");
    return QASR_ERR_INVALID;
  }
  const int64_t target = (int64_t)(segment_sec * 16000.0f);
  const float search = std::min(search_sec, segment_sec / 2.0f);
  const int64_t margin = (int64_t)(search * 16000.0f);
  std::vector<int64_t> splits = {0};
  if (segment_sec > 0.0f && n > target + margin) {
    int64_t pos = 0;
    while (pos + target + margin < n) {
      const int64_t split = qasr_find_split_point(samples, n, pos + target, search);
      splits.push_back(split);
      pos = split;
      if (splits.size() >= 127) break;
    }
  }
  *n_segments = (int)splits.size();
  std::memcpy(starts, splits.data(), sizeof(int64_t) * std::min<size_t>(cap, splits.size()));
  return QASR_OK;
}
