"""Restatement of the reference's streaming transcription
(crates/qwen-asr/src/transcribe.rs: transcribe_stream 445-800, StreamState +
stream_push_audio 809-1495) over the CPU oracle decoder, for the streaming
parity tests.  The encoder is a callback (samples -> rows), so a test can
feed the device encoder's rows and compare the decoder-side bookkeeping
exactly.  Test infrastructure only.
"""
from __future__ import annotations

import numpy as np

from qwenasr_b200.transcribe import PREFIX_HEAD, PREFIX_TAIL, SUFFIX_BASE

EOT, IM_END, ASR_TEXT = 151643, 151645, 151704
DEGEN_MAX_PERIOD, DEGEN_MIN_REPEATS, STALE_CHUNKS = 6, 4, 4
RESET_INTERVAL, CARRY, REANCHOR_ROWS = 45, 24, 200


def tail_repeat_blocks(tokens, max_period):
    """stream_tail_repeat_blocks (transcribe.rs:42-59)."""
    n = len(tokens)
    if n < 2:
        return 1, 0
    cap = min(n // 2, max_period if max_period > 0 else n // 2)
    best, best_p = 1, 0
    for p in range(1, cap + 1):
        reps = 1
        while (reps + 1) * p <= n and tokens[n - (reps + 1) * p:n - reps * p] == tokens[n - reps * p:n - (reps - 1) * p]:
            reps += 1
        if reps > best:
            best, best_p = reps, p
    return best, best_p


def find_split_point(samples, target, search_sec):
    """find_split_point (transcribe.rs:250-275) with f32 sums in order."""
    half = int(np.float32(search_sec) * np.float32(16000.0))
    lo = max(target - half, 0)
    hi = min(target + half, len(samples))
    win, best, center, pos = 1600, np.float32(1e30), target, lo
    while pos + win <= hi:
        end = min(pos + win, len(samples))
        e = np.float32(0.0)
        for j in range(pos, end):
            e = np.float32(e + np.float32(samples[j] * samples[j]))
        e = np.float32(e / np.float32(end - pos))
        if e < best:
            best, center = e, pos + (end - pos) // 2
        pos += win // 2
    return center


class OracleStream:
    def __init__(self, od, embed, encode, max_seq, chunk_sec=2.0, rollback=5, unfixed_chunks=2, max_new_tokens=32,
                 past_text_conditioning=False, incremental=True, prompt=(), force=(), tok_bytes=None,
                 window_frames=800):
        self.od, self.embed, self.encode, self.max_seq = od, embed, encode, max_seq
        self.chunk = int(np.float32(chunk_sec) * np.float32(16000.0))
        self.rollback, self.unfixed, self.max_new = rollback, unfixed_chunks, max_new_tokens or 32
        self.past, self.incremental = past_text_conditioning, incremental
        self.prompt, self.force = list(prompt), list(force)
        self.tok_bytes = tok_bytes
        self.window = min(800, max(100, window_frames)) * 160
        self.enc_cache, self.enc_total, self.base = [], 0, 0
        self.raw, self.stable, self.emitted = [], [], []
        self.prev_rows, self.prev_len = None, 0
        self.snapshot, self.stale = [], 0
        self.last_partial_cursor, self.last_partial = 0, None
        self.cursor, self.chunk_idx, self.trim_request = 0, 0, 0
        self.max_prefix, self.resets, self.max_reused = 0, 0, 0  # coverage counters for the tests
        self.k, self.v = od.new_kv(max_seq)

    def _bytes(self, t):
        return int(self.tok_bytes[t]) if self.tok_bytes is not None and 0 <= t < len(self.tok_bytes) else 1

    def _reset_tokens(self, keep_windows):
        self.resets += 1
        carry = min(len(self.stable), CARRY)
        carried = self.stable[len(self.stable) - carry:]
        self.raw = ([ASR_TEXT] + carried) if carry else []
        self.stable = list(carried)
        self.prev_rows, self.prev_len = None, 0
        self.stale, self.snapshot = 0, []
        keep = min(keep_windows, len(self.enc_cache))
        drop = len(self.enc_cache) - keep
        if drop:
            self.enc_total = max(0, self.enc_total - sum(len(w) for w in self.enc_cache[:drop]))
            self.base += drop
            self.enc_cache = self.enc_cache[drop:]
        if self.incremental and self.cursor > self.chunk * 4:
            self.trim_request = self.cursor - self.chunk * 4

    def push(self, samples, finalize=True):
        samples = np.asarray(samples, np.float32)
        n, delta = len(samples), []
        if self.incremental:
            avail = max(n - self.cursor, 0)
            if (avail < self.chunk and not finalize) or avail == 0:
                return []
        while self.cursor < n:
            if self.incremental and n - self.cursor < self.chunk and not finalize:
                break
            self.cursor = min(self.cursor + self.chunk, n)
            is_final = (finalize and self.cursor >= n) if self.incremental else self.cursor >= n
            full_end = (self.cursor // self.window) * self.window
            while (self.base + len(self.enc_cache)) * self.window < full_end:
                ws = (self.base + len(self.enc_cache)) * self.window
                rows = self.encode(samples[ws:ws + self.window])
                self.enc_total += len(rows)
                self.enc_cache.append(rows)
            partial = None
            if full_end < self.cursor:
                if self.incremental:
                    need = (self.last_partial_cursor == 0 or self.cursor - self.last_partial_cursor >= 2 * self.chunk
                            or is_final)
                    if need and (self.cursor - full_end) // 160 > 0:
                        partial = self.encode(samples[full_end:self.cursor])
                        self.last_partial_cursor, self.last_partial = self.cursor, partial
                    else:
                        partial = self.last_partial
                elif (self.cursor - full_end) // 160 > 0:
                    partial = self.encode(samples[full_end:self.cursor])
            n_partial = 0 if partial is None else len(partial)
            enc_rows = self.enc_total + n_partial
            if enc_rows == 0:
                self.chunk_idx += 1
                if self.incremental:
                    return []
                continue
            n_prefix = (max(len(self.raw) - self.rollback, 0)
                        if self.past and self.chunk_idx >= self.unfixed and self.raw else 0)
            self.max_prefix = max(self.max_prefix, n_prefix)
            pre = list(PREFIX_HEAD) + self.prompt + list(PREFIX_TAIL)
            post = list(SUFFIX_BASE) + self.force + self.raw[:n_prefix]
            parts = [self.embed(pre)] + self.enc_cache + ([partial] if n_partial else []) + [self.embed(post)]
            rows = np.concatenate(parts).astype(np.float32)
            prefill_len = len(rows) - 1
            reused = 0
            if self.prev_rows is not None and self.prev_len > 0:
                cmp = min(prefill_len, self.prev_len)
                while reused < cmp and np.array_equal(self.prev_rows[reused], rows[reused]):
                    reused += 1
            self.max_reused = max(self.max_reused, reused)
            if prefill_len > reused:
                self.od.prefill(self.k, self.v, reused, rows[reused:prefill_len])
            tok = post[-1]
            self.prev_rows, self.prev_len = rows[:prefill_len].copy(), prefill_len
            chunk_tokens, pos = [], prefill_len
            tok, _, _ = self.od.forward(self.k, self.v, pos, rows[prefill_len])
            for _ in range(self.max_new):
                if tok in (EOT, IM_END):
                    break
                chunk_tokens.append(tok)
                if len(chunk_tokens) == self.max_new:
                    break  # the reference's extra step after the last token changes no id
                pos += 1
                tok, _, _ = self.od.forward(self.k, self.v, pos, self.embed([tok])[0])
            self.raw = self.raw[:n_prefix] + chunk_tokens
            if self.raw == self.snapshot:
                self.stale += 1
            else:
                self.stale, self.snapshot = 0, list(self.raw)
            reps, _ = tail_repeat_blocks(self.raw, DEGEN_MAX_PERIOD)
            if self.stale >= STALE_CHUNKS or reps >= DEGEN_MIN_REPEATS:
                self._reset_tokens(1 if self.incremental else 2)
            if (self.chunk_idx > 0 and self.chunk_idx % RESET_INTERVAL == 0) or enc_rows >= REANCHOR_ROWS:
                self._reset_tokens(1)
            text_start = self.raw.index(ASR_TEXT) + 1 if ASR_TEXT in self.raw else 0
            cand = self.raw[text_start:]
            if is_final:
                cand_len = len(cand)
            elif self.chunk_idx >= self.unfixed:
                cand_len = max(len(cand) - self.rollback, 0)
            else:
                cand_len = 0
            emit_from = len(self.stable)
            emit_to = max(cand_len, emit_from)
            if self.incremental and emit_from > 0:
                mm = None
                for j in range(min(emit_from, len(cand))):
                    if j < len(self.stable) and self.stable[j] != cand[j]:
                        mm = j
                        break
                if mm is None and len(self.stable) > len(cand):
                    mm = len(cand)
                if mm is not None:
                    target = sum(self._bytes(t) for t in self.stable[:mm])
                    aligned, cum = len(cand), 0
                    for j, t in enumerate(cand):
                        cum += self._bytes(t)
                        if cum >= target:
                            aligned = j + 1
                            break
                    aligned = min(aligned, len(cand))
                    self.stable = list(cand[:aligned])
                    emit_from = aligned
                    emit_to = max(cand_len, emit_from)
            for i in range(emit_from, emit_to):
                if i < len(cand):
                    if i >= len(self.stable):
                        self.stable.append(cand[i])
                    delta.append(cand[i])
                    self.emitted.append(cand[i])
            self.chunk_idx += 1
        return delta
