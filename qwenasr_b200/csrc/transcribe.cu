// transcribe.cu -- transcribe_segment (crates/qwen-asr/src/transcribe.rs:67-244)
// on the device, token ids out (the host keeps its tokenizer):
//
//   samples -> qasr_mel_spectrogram -> qasr_encoder_forward -> prompt
//   embeddings (PREFIX_HEAD, prompt, PREFIX_TAIL, audio rows, SUFFIX_BASE,
//   forced tokens; transcribe.rs:11-13, 98-170) -> qasr_decoder_prefill of
//   all but the last prompt row -> greedy decode from the last prompt token.
//
// Up to max_batch independent segments run together (the segmented mode,
// transcribe.rs:354-420, with past_text_conditioning off): each is encoded
// and prefilled into its own KV slot, then all decode in one batched step.
// The decode loop keeps the ids on the device: step s reads step s-1's
// argmax as its tokens and a precomputed position row, so consecutive steps
// are enqueued back to back with no host round trip; the host looks at the
// ids only every kCheckEvery steps, when stopping at end-of-text.
#include <algorithm>
#include <atomic>
#include <cstring>
#include <exception>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "common.cuh"
#include "engine.cuh"
#include "matvec.cuh"
#include "qwenasr_cuda.h"

namespace qasr {

// transcribe.rs:11-13
const int32_t kPrefixHead[3] = {151644, 8948, 198};
const int32_t kPrefixTail[6] = {151645, 198, 151644, 872, 198, 151669};
const int32_t kSuffixBase[6] = {151670, 151645, 198, 151644, 77091, 198};

namespace {
constexpr int kHead = 3, kTail = 6, kSuffix = 6;
constexpr int kCheckEvery = 32;
}  // namespace

bool is_stop_token(int32_t t) { return t == kTokEndOfText || t == kTokImEnd; }

int encode_samples(qasr_encoder *enc, int device, cudaStream_t st, const float *samples, int n_samples, float *rows,
                   int rows_cap, int *T) {
  const int frames = qasr_mel_frames(n_samples);
  if (frames <= 0) {
    set_error("encode: %d samples (at least 160 needed)", n_samples);
    return QASR_ERR_INVALID;
  }
  void *audio = nullptr, *mel = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchAudio, (size_t)n_samples * 4, &audio))) return rc;
  if ((rc = dev_scratch(kScratchMelOut, (size_t)128 * frames * 4, &mel))) return rc;
  if ((rc = cuda_status(cudaMemcpyAsync(audio, samples, (size_t)n_samples * 4, cudaMemcpyDefault, st),
                        "encode: samples")))
    return rc;
  if ((rc = qasr_mel_spectrogram(static_cast<float *>(mel), static_cast<const float *>(audio), n_samples, st)))
    return rc;
  if ((rc = cuda_status(cudaStreamSynchronize(st), "encode: mel"))) return rc;
  rc = qasr_encoder_forward(enc, static_cast<const float *>(mel), frames, rows, rows_cap, T);
  cudaSetDevice(device);
  return rc;
}

// Greedy decode of M sequences (KV slots 0..M-1) from token tok0[i] at
// position pos0[i]: the ids stay on the device, step s reading step s-1's
// argmax, so steps are enqueued back to back; the host reads the ids every
// check_every steps when stopping at end-of-text (the stop token is kept).
int greedy_decode(qasr_decoder *dec, int M, const int32_t *tok0, const int32_t *pos0, int max_new, int stop_at_eos,
                  int check_every, int32_t *ids, int ids_stride, int *n_ids) {
  cudaStream_t st = reinterpret_cast<cudaStream_t>(qasr_decoder_stream(dec));
  void *steps = nullptr;
  int rc = dev_scratch(kScratchDecode, (size_t)(M + 2 * (size_t)max_new * M) * 4, &steps);
  if (rc) return rc;
  int32_t *d_tok0 = static_cast<int32_t *>(steps), *d_pos = d_tok0 + M, *d_ids = d_pos + (size_t)max_new * M;
  std::vector<int32_t> pos((size_t)max_new * M);
  for (int s = 0; s < max_new; ++s)
    for (int i = 0; i < M; ++i) pos[(size_t)s * M + i] = pos0[i] + s;
  if ((rc = cuda_status(cudaMemcpyAsync(d_tok0, tok0, (size_t)M * 4, cudaMemcpyHostToDevice, st), "decode: tokens")))
    return rc;
  if ((rc = cuda_status(cudaMemcpyAsync(d_pos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice, st),
                        "decode: positions")))
    return rc;
  std::vector<int32_t> out((size_t)max_new * M);
  std::vector<int> count(M, 0);
  std::vector<char> done(M, 0);
  int steps_run = 0;
  while (steps_run < max_new) {
    const int upto = std::min(max_new, steps_run + (stop_at_eos ? check_every : max_new));
    for (int s = steps_run; s < upto; ++s) {
      const int32_t *tok = s == 0 ? d_tok0 : d_ids + (size_t)(s - 1) * M;
      if ((rc = qasr_decoder_step_device(dec, tok, d_pos + (size_t)s * M, M, d_ids + (size_t)s * M))) return rc;
    }
    if ((rc = cuda_status(cudaMemcpyAsync(out.data() + (size_t)steps_run * M, d_ids + (size_t)steps_run * M,
                                          (size_t)(upto - steps_run) * M * 4, cudaMemcpyDeviceToHost, st),
                          "decode: ids")))
      return rc;
    if ((rc = cuda_status(cudaStreamSynchronize(st), "decode"))) return rc;
    for (int s = steps_run; s < upto; ++s)
      for (int i = 0; i < M; ++i) {
        if (done[i]) continue;
        const int32_t t = out[(size_t)s * M + i];
        ids[(size_t)i * ids_stride + count[i]++] = t;
        if (stop_at_eos && is_stop_token(t)) done[i] = 1;
      }
    steps_run = upto;
    if (std::all_of(done.begin(), done.end(), [](char c) { return c != 0; })) break;
  }
  std::memcpy(n_ids, count.data(), (size_t)M * sizeof(int));
  return QASR_OK;
}

}  // namespace qasr

using namespace qasr;

extern "C" int qasr_transcribe_prompt_len(int n_audio_tokens, int n_prompt, int n_force) {
  if (n_audio_tokens < 0 || n_prompt < 0 || n_force < 0) return 0;
  return kHead + n_prompt + kTail + n_audio_tokens + kSuffix + n_force;
}

extern "C" int qasr_transcribe_batch(qasr_decoder *dec, qasr_encoder *enc, const float *const *samples,
                                     const int *n_samples, int n_segments, const int32_t *prompt_tokens, int n_prompt,
                                     const int32_t *force_tokens, int n_force, int max_new, int stop_at_eos,
                                     int32_t *ids, int ids_stride, int *n_ids) {
  const qasr_decoder_config *dc = qasr_decoder_get_config(dec);
  const qasr_encoder_config *ec = qasr_encoder_get_config(enc);
  if (!dc || !ec || !samples || !n_samples || !ids || !n_ids || n_segments <= 0 || n_segments > dc->max_batch ||
      max_new <= 0 || ids_stride < max_new || n_prompt < 0 || n_force < 0 || (n_prompt && !prompt_tokens) ||
      (n_force && !force_tokens)) {
    set_error("qasr_transcribe_batch: invalid arguments (%d segments, max_new %d)", n_segments, max_new);
    return QASR_ERR_INVALID;
  }
  if (ec->output_dim != dc->hidden) {
    set_error("qasr_transcribe_batch: encoder output %d != decoder hidden %d", ec->output_dim, dc->hidden);
    return QASR_ERR_INVALID;
  }
  const int dev = qasr_decoder_device(dec);
  if (qasr_encoder_device(enc) != dev) {
    set_error("qasr_transcribe_batch: encoder on device %d, decoder on device %d", qasr_encoder_device(enc), dev);
    return QASR_ERR_INVALID;
  }
  if (int rc = cuda_status(cudaSetDevice(dev), "qasr_transcribe_batch")) return rc;
  ArenaScope arena_scope(decoder_arena(dec));
  const int H = dc->hidden, M = n_segments;
  int max_samples = 0, max_tokens = 0;
  for (int i = 0; i < M; ++i) {
    const int frames = qasr_mel_frames(n_samples[i]);
    if (!samples[i] || frames <= 0) {
      set_error("qasr_transcribe_batch: segment %d has %d samples (at least 160 needed)", i, n_samples[i]);
      return QASR_ERR_INVALID;
    }
    max_samples = std::max(max_samples, n_samples[i]);
    max_tokens = std::max(max_tokens, qasr_encoder_tokens(enc, frames));
    const int total = qasr_transcribe_prompt_len(qasr_encoder_tokens(enc, frames), n_prompt, n_force);
    if (total - 1 + max_new > dc->max_seq) {
      set_error("qasr_transcribe_batch: segment %d needs %d positions, the cache holds %d", i, total - 1 + max_new,
                dc->max_seq);
      return QASR_ERR_INVALID;
    }
  }
  const int max_prompt = qasr_transcribe_prompt_len(max_tokens, n_prompt, n_force);
  cudaStream_t st = reinterpret_cast<cudaStream_t>(qasr_decoder_stream(dec));
  // every segment's log-mel, then one encoder pass over all of them (transcribe.rs:78-96)
  std::vector<int> frames(M), tokens(M), tok_off(M + 1, 0);
  std::vector<size_t> mel_off(M + 1, 0);
  for (int i = 0; i < M; ++i) {
    frames[i] = qasr_mel_frames(n_samples[i]);
    mel_off[i + 1] = mel_off[i] + (size_t)128 * frames[i];
    tokens[i] = qasr_encoder_tokens(enc, frames[i]);
    tok_off[i + 1] = tok_off[i] + tokens[i];
  }
  void *audio = nullptr, *mel = nullptr, *enc_out = nullptr, *prompt = nullptr;
  int rc;
  if ((rc = dev_scratch(kScratchAudio, (size_t)max_samples * 4, &audio))) return rc;
  if ((rc = dev_scratch(kScratchMelOut, mel_off[M] * 4, &mel))) return rc;
  if ((rc = dev_scratch(kScratchEncOut, (size_t)tok_off[M] * H * 4, &enc_out))) return rc;
  // prompt rows of every segment, side by side (one batched prefill)
  if ((rc = dev_scratch(kScratchPrompt, (size_t)M * max_prompt * H * 4, &prompt))) return rc;
  std::vector<const float *> mels(M);
  std::vector<float *> outs(M);
  for (int i = 0; i < M; ++i) {
    float *m = static_cast<float *>(mel) + mel_off[i];
    if ((rc = cuda_status(cudaMemcpyAsync(audio, samples[i], (size_t)n_samples[i] * 4, cudaMemcpyDefault, st),
                          "qasr_transcribe_batch: samples")))
      return rc;
    if ((rc = qasr_mel_spectrogram(m, static_cast<const float *>(audio), n_samples[i], st))) return rc;
    mels[i] = m;
    outs[i] = static_cast<float *>(enc_out) + (size_t)tok_off[i] * H;
  }
  if ((rc = cuda_status(cudaStreamSynchronize(st), "qasr_transcribe_batch: mel"))) return rc;
  std::vector<int> got(M);
  if ((rc = qasr_encoder_forward_batch(enc, mels.data(), frames.data(), M, outs.data(), tokens.data(), got.data())))
    return rc;
  cudaSetDevice(dev);
  std::vector<int32_t> tok0(M), pos0(M), pre;
  std::vector<int> slots(M), lens(M), starts(M, 0);
  std::vector<const float *> rows_of(M);
  for (int i = 0; i < M; ++i) {
    float *embeds = static_cast<float *>(prompt) + (size_t)i * max_prompt * H;
    const int T = got[i];
    const float *rows_i = outs[i];
    // prompt embeddings (transcribe.rs:98-170): token rows around the audio rows
    pre.assign(kPrefixHead, kPrefixHead + kHead);
    pre.insert(pre.end(), prompt_tokens, prompt_tokens + n_prompt);
    pre.insert(pre.end(), kPrefixTail, kPrefixTail + kTail);
    const int prefix_len = (int)pre.size();
    std::vector<int32_t> post(kSuffixBase, kSuffixBase + kSuffix);
    post.insert(post.end(), force_tokens, force_tokens + n_force);
    const int total = prefix_len + T + (int)post.size();
    if ((rc = qasr_decoder_embed(dec, pre.data(), prefix_len, embeds))) return rc;
    if ((rc = cuda_status(cudaMemcpyAsync(embeds + (size_t)prefix_len * H, rows_i, (size_t)T * H * 4,
                                          cudaMemcpyDeviceToDevice, st),
                          "qasr_transcribe_batch: audio rows")))
      return rc;
    if ((rc = qasr_decoder_embed(dec, post.data(), (int)post.size(), embeds + (size_t)(prefix_len + T) * H)))
      return rc;
    // prefill all but the last row; the first decode step feeds the last
    // prompt token at position total - 1 (transcribe.rs:172-190)
    slots[i] = i;
    lens[i] = total - 1;
    rows_of[i] = embeds;
    tok0[i] = post.back();
    pos0[i] = total - 1;
  }
  if ((rc = qasr_decoder_prefill_batch(dec, slots.data(), rows_of.data(), lens.data(), starts.data(), M))) return rc;
  // greedy decode (transcribe.rs:192-222)
  return greedy_decode(dec, M, tok0.data(), pos0.data(), max_new, stop_at_eos, kCheckEvery, ids, ids_stride, n_ids);
}


// Independent segments over several engine lanes: transcribe_audio's
// segment loop (transcribe.rs:354-420, past_text_conditioning off, so no
// segment depends on another) with the segments taken in batches by
// whichever lane is free.  Each lane is one decoder + encoder pair driven by
// its own host thread (the first by the caller's): the engines have their
// own streams, graphs and scratch, so one lane's encoder and prefill overlap
// another lane's latency-bound decode steps on the same GPU, and lanes on
// different GPUs run side by side.  Batches are full (the smallest lane's
// max_batch): a decode step costs about the same at 4 sequences as at 8, so
// splitting one batch over two lanes would double the weight traffic for
// the same tokens (measured: 8 segments over two lanes of 4 run 17 % slower
// than one batch of 8).  Per-segment results equal qasr_transcribe_batch's, as every
// kernel on the path is row-independent.
extern "C" int qasr_transcribe_lanes(qasr_decoder *const *decs, qasr_encoder *const *encs, int n_lanes,
                                     const float *const *samples, const int *n_samples, int n_segments,
                                     const int32_t *prompt_tokens, int n_prompt, const int32_t *force_tokens,
                                     int n_force, int max_new, int stop_at_eos, int32_t *ids, int ids_stride,
                                     int *n_ids) {
  if (!decs || !encs || n_lanes <= 0 || n_lanes > 64 || n_segments < 0 || (n_segments && (!samples || !n_samples)) ||
      !ids || !n_ids || max_new <= 0 || ids_stride < max_new) {
    set_error("qasr_transcribe_lanes: invalid arguments (%d lanes, %d segments)", n_lanes, n_segments);
    return QASR_ERR_INVALID;
  }
  int batch = 1 << 30;
  for (int l = 0; l < n_lanes; ++l) {
    const qasr_decoder_config *dc = qasr_decoder_get_config(decs[l]);
    if (!dc || !qasr_encoder_get_config(encs[l])) {
      set_error("qasr_transcribe_lanes: lane %d has no decoder or encoder", l);
      return QASR_ERR_INVALID;
    }
    for (int j = 0; j < l; ++j)
      if (decs[j] == decs[l] || encs[j] == encs[l]) {
        set_error("qasr_transcribe_lanes: lanes %d and %d share an engine", j, l);
        return QASR_ERR_INVALID;
      }
    batch = std::min(batch, dc->max_batch);
  }
  if (n_segments == 0) return QASR_OK;
  const int n_batches = (n_segments + batch - 1) / batch;
  std::atomic<int> next{0};
  std::atomic<bool> failed{false};
  std::mutex mu;
  int first_rc = QASR_OK;
  std::string first_msg;
  auto lane = [&](int l) {
    for (;;) {
      if (failed.load()) return;
      const int b = next.fetch_add(1);
      if (b >= n_batches) return;
      const int lo = b * batch, cnt = std::min(batch, n_segments - lo);
      int rc;
      try {  // an exception must not leave a lane thread (std::terminate)
        rc = qasr_transcribe_batch(decs[l], encs[l], samples + lo, n_samples + lo, cnt, prompt_tokens, n_prompt,
                                   force_tokens, n_force, max_new, stop_at_eos, ids + (size_t)lo * ids_stride,
                                   ids_stride, n_ids + lo);
      } catch (const std::exception &ex) {
        set_error("host exception: %s", ex.what());
        rc = QASR_ERR_ALLOC;
      } catch (...) {
        set_error("host exception");
        rc = QASR_ERR_INVALID;
      }
      if (rc) {
        std::lock_guard<std::mutex> lk(mu);
        if (!first_rc) {
          first_rc = rc;
          first_msg = std::string("lane ") + std::to_string(l) + ": " + qasr_last_error();
        }
        failed.store(true);
        return;
      }
    }
  };
  std::vector<std::thread> threads;
  const int use = std::min(n_lanes, n_batches);
  for (int l = 1; l < use; ++l) {
    try {
      threads.emplace_back(lane, l);
    } catch (...) {
      break;  // fewer threads: the running lanes take the remaining batches
    }
  }
  lane(0);
  for (auto &t : threads) t.join();
  if (first_rc) set_error("qasr_transcribe_lanes: %s", first_msg.c_str());
  return first_rc;
}
