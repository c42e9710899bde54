// engine.cuh -- pieces of the transcription path shared by the offline
// (transcribe.cu) and streaming (stream.cu) drivers.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qwenasr_cuda.h"

namespace qasr {

// transcribe.rs:11-13 and config.rs:13-19
extern const int32_t kPrefixHead[3], kPrefixTail[6], kSuffixBase[6];
constexpr int32_t kTokEndOfText = 151643, kTokImEnd = 151645, kTokAsrText = 151704;

bool is_stop_token(int32_t t);

// Greedy decode of M sequences in KV slots 0..M-1 from tok0[i] at pos0[i]
// (host arrays); ids[i * ids_stride + j], n_ids[i] (stop token kept when
// stop_at_eos).
int greedy_decode(qasr_decoder *dec, int M, const int32_t *tok0, const int32_t *pos0, int max_new, int stop_at_eos,
                  int check_every, int32_t *ids, int ids_stride, int *n_ids);

// samples (host or device) -> log-mel -> encoder rows [T, output_dim] into
// rows (device, rows_cap rows).  Runs on stream st (synchronised) and the
// encoder's own stream.  Leaves `device` current.
int encode_samples(qasr_encoder *enc, int device, cudaStream_t st, const float *samples, int n_samples, float *rows,
                   int rows_cap, int *T);

}  // namespace qasr
