"""Per-stream restatement of the reference's streaming loop - TEST INFRASTRUCTURE.

Only tests/ and bench.py's reference arm may import this module; it checks
qdb_streams_* (qwen-asr_b200/csrc/qdb_stream.cu) and is never the product.

Restates the decoder side of stream_impl (qwen_asr.c, reference project), one
stream at a time in the reference's own order, one qwen_decoder_* call at a
time:
  prefix rollback                  :1676-1690 (QWEN_STREAM_MAX_PREFIX_TOKENS 150)
  prompt embeddings                :1692-1746 [head][prompt][tail][audio][suffix][force][prefix]
  prefill-KV reuse by memcmp       :1748-1770 (kv_cache_len = reused prefix, prefill the delta)
  first token + decode loop        :1772-1829 (<= max_new_tokens, stop at an end token)
  repeat-run suppression           :1850-1884 (runs > 12 dropped)
  raw history update               :1886-1906
  text region after <asr_text>     :1908-1922
  fixed frontier                   :1924-1941
  recovery resets                  :1943-1992 (stream_tail_repeat_blocks :1078-1111)
  commit + overlap de-duplication  :1993-2054
  periodic re-anchor               :2057-2085 (stream_reanchor_text_state :1135-1182)
The decoder is any object with prefill(embeds, start_pos) and
forward(embed_row, pos) -> (token, logits or None); embed(token) -> f32 row.
Prompt rows are compared with memcmp semantics (bytes of the f32 rows).
"""
from __future__ import annotations

import numpy as np

MAX_PREFIX_TOKENS = 150
MAX_REPEAT_TOKEN_RUN = 12
OVERLAP_MAX_TOKENS = 48
OVERLAP_MIN_TOKENS = 4
DEGEN_MAX_PERIOD = 6
DEGEN_MIN_REPEATS = 4
STALE_CHUNKS = 4
RESET_INTERVAL_CHUNKS = 45
RESET_CARRY_TOKENS = 24
TOKEN_ENDOFTEXT, TOKEN_IM_END, TOKEN_ASR_TEXT = 151643, 151645, 151704
HEAD = [151644, 8948, 198]
TAIL = [151645, 198, 151644, 872, 198, 151669]
SUFFIX = [151670, 151645, 198, 151644, 77091, 198]


def tail_repeat_blocks(tokens, max_period):
    """(reps, period) of the longest repeated block at the end (qwen_asr.c:1078-1111)."""
    n = len(tokens)
    if n < 2:
        return 1, 0
    best, best_p = 1, 0
    cap = n // 2
    if max_period > 0 and cap > max_period:
        cap = max_period
    for p in range(1, cap + 1):
        reps = 1
        while (reps + 1) * p <= n and tokens[n - (reps + 1) * p:n - reps * p] == tokens[n - reps * p:n - (reps - 1) * p]:
            reps += 1
        if reps > best:
            best, best_p = reps, p
    return best, best_p


class StreamOracle:
    def __init__(self, decoder, embed, max_new_tokens=32, rollback=5, unfixed_chunks=2, past_text=False,
                 head=None, tail=None, suffix=None, prompt=None, force=None, asr_text_token=TOKEN_ASR_TEXT):
        self.dec, self.embed = decoder, embed
        self.max_new, self.rollback, self.unfixed, self.past_text = max_new_tokens, rollback, unfixed_chunks, past_text
        self.head = list(HEAD if head is None else head)
        self.tail = list(TAIL if tail is None else tail)
        self.suffix = list(SUFFIX if suffix is None else suffix)
        self.prompt = list(prompt or [])
        self.force = list(force or [])
        self.asr_text = asr_text_token
        self.chunk_idx = 0
        self.raw, self.stable, self.emitted = [], [], []
        self.stagnant = 0
        self.prev = None  # previous prefill rows (prev_prefill_embeds[:prev_prefill_len])
        self.kv_len = 0
        self.prefill_total = self.prefill_reused = 0
        self.min_margin = np.inf
        self.last = {}

    def _forward(self, row):
        tok, logits = self.dec.forward(row, self.kv_len)
        self.kv_len += 1
        if logits is not None:
            l = np.sort(logits.astype(np.float64))
            self.min_margin = min(self.min_margin, float(l[-1] - l[-2]))
        return tok

    def _reanchor(self):
        carry = min(len(self.emitted), RESET_CARRY_TOKENS)
        lead = [self.asr_text] if not self.force else []
        tail = self.emitted[len(self.emitted) - carry:]
        self.raw = lead + list(tail)
        self.stable = list(tail)

    def chunk(self, audio, is_final):
        """One chunk; audio = f32 [rows, hidden] encoder output (None / 0 rows:
        the chunk is skipped). Returns (n_emitted, reset)."""
        self.last = {}
        if audio is None or len(audio) == 0:
            self.chunk_idx += 1
            return 0, 0
        n_full = n_pref = off = 0
        if self.past_text and self.chunk_idx >= self.unfixed and self.raw:
            n_full = max(0, len(self.raw) - self.rollback)
            n_pref = min(n_full, MAX_PREFIX_TOKENS)
            off = n_full - n_pref
        rows = [self.embed(t) for t in self.head + self.prompt + self.tail]
        rows += [np.asarray(r, np.float32) for r in audio]
        rows += [self.embed(t) for t in self.suffix + self.force + self.raw[off:off + n_pref]]
        emb = np.stack(rows).astype(np.float32)
        prefill_len = len(emb) - 1
        reused = 0
        if self.prev is not None and len(self.prev) > 0:
            cmp = min(prefill_len, len(self.prev))
            while reused < cmp and emb[reused].tobytes() == self.prev[reused].tobytes():
                reused += 1
        self.kv_len = reused
        if prefill_len - reused > 0:
            self.dec.prefill(emb[reused:prefill_len], reused)
            self.kv_len = prefill_len
        self.prefill_total += prefill_len
        self.prefill_reused += reused
        token = self._forward(emb[prefill_len])
        self.prev = emb[:prefill_len].copy()
        chunk, n_gen = [], 0
        while n_gen < self.max_new:
            n_gen += 1
            if token in (TOKEN_ENDOFTEXT, TOKEN_IM_END):
                break
            chunk.append(token)
            if n_gen < self.max_new:  # the reference's last forward's token is never read
                token = self._forward(self.embed(token))
        self.last.update(reused=reused, prefill_len=prefill_len, generated=n_gen)
        # repeat-run suppression
        dropped = 0
        if chunk:
            prev_tok, prev_run = -1, 0
            if n_full > 0:
                prev_tok, prev_run = self.raw[n_full - 1], 1
                for j in range(n_full - 2, -1, -1):
                    if self.raw[j] != prev_tok:
                        break
                    prev_run += 1
                    if prev_run >= MAX_REPEAT_TOKEN_RUN:
                        break
            kept = []
            for t in chunk:
                if t == prev_tok:
                    prev_run += 1
                    if prev_run > MAX_REPEAT_TOKEN_RUN:
                        dropped += 1
                        continue
                else:
                    prev_tok, prev_run = t, 1
                kept.append(t)
            chunk = kept
        self.raw = self.raw[:n_full] + chunk
        text_start = 0
        if not self.force:
            text_start = self.raw.index(self.asr_text) + 1 if self.asr_text in self.raw else 0
        n_text = len(self.raw) - text_start
        if is_final:
            cand = n_text
        elif self.chunk_idx >= self.unfixed:
            cand = n_text - self.rollback
            if cand <= 0 and n_text > 0:
                cand = n_text - 1
            cand = max(cand, 0)
        else:
            cand = 0
        cand_tok = self.raw[text_start:text_start + cand]
        reps, period = tail_repeat_blocks(cand_tok, DEGEN_MAX_PERIOD)
        advance = cand - len(self.stable)
        self.stagnant = self.stagnant + 1 if (not is_final and n_gen >= self.max_new and advance <= 1) else 0
        recovery = (period > 0 and reps >= DEGEN_MIN_REPEATS) or self.stagnant >= STALE_CHUNKS or dropped >= 8
        n_emit, reset = 0, 0
        if recovery:
            self._reanchor()
            self.prev = None
            self.stagnant = 0
            reset = 1
        else:
            lcp = 0
            while lcp < len(self.stable) and lcp < cand and self.stable[lcp] == cand_tok[lcp]:
                lcp += 1
            self.stable = self.stable[:lcp] + cand_tok[lcp:]
            emit_start = lcp
            if emit_start < cand and self.emitted:
                max_ov = min(cand - emit_start, len(self.emitted), OVERLAP_MAX_TOKENS)
                for k in range(max_ov, OVERLAP_MIN_TOKENS - 1, -1):
                    if self.emitted[-k:] == cand_tok[emit_start:emit_start + k]:
                        emit_start += k
                        break
            new = self.stable[emit_start:cand]
            self.emitted += new
            n_emit = len(new)
            self.stable = self.stable[:cand]
            if (not is_final and self.past_text and self.chunk_idx >= self.unfixed
                    and (self.chunk_idx + 1) % RESET_INTERVAL_CHUNKS == 0):
                self._reanchor()
                self.prev = None
                reset = 2
        self.chunk_idx += 1
        return n_emit, reset
