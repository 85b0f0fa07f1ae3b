"""qwen-asr_b200: B200 decoder hot path of qwen-asr behind a C ABI.

Host-side Python mirror of the reference decoder interface
(qwen_decoder_prefill / qwen_decoder_forward, qwen_asr.h:313-317) over
libqwen_asr_b200.so (include/qwen_asr_b200.h). The CUDA library is the only
compute path: importing this package fails loudly when the library is missing,
and there is no CPU fallback.

    ctx = Decoder(model, capacity)      # one utterance: device KV cache
    ctx.kv_cache_len = 0                # host-owned length, as qwen_ctx_t
    ctx.prefill(input_embeds)           # appends len(input_embeds) positions
    tok = ctx.forward(embed)            # one position, returns greedy token
"""
from __future__ import annotations

import atexit
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
# QWEN_ASR_B200_LIB selects another build of the same library (A/B runs of
# compile-time variants); the default is the in-tree build.
LIB_PATH = os.environ.get("QWEN_ASR_B200_LIB") or os.path.join(_HERE, "libqwen_asr_b200.so")

QWEN_TOKEN_ENDOFTEXT = 151643
QWEN_TOKEN_IM_END = 151645

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i32p = ctypes.POINTER(ctypes.c_int)


class QdbConfig(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("layers", ctypes.c_int), ("heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("intermediate", ctypes.c_int),
                ("vocab", ctypes.c_int), ("eps", ctypes.c_float), ("theta", ctypes.c_float)]


# Every symbol include/qwen_asr_b200.h declares: name -> (restype, argtypes).
ABI = {
    "qdb_last_error": (ctypes.c_char_p, []),
    "qdb_device_count": (ctypes.c_int, []),
    "qdb_model_create": (ctypes.c_void_p, [ctypes.POINTER(QdbConfig), ctypes.c_int]),
    "qdb_model_set_embed": (ctypes.c_int, [ctypes.c_void_p, _u16p, _f32p]),
    "qdb_model_set_layer": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int] + [_u16p] * 7 + [_f32p] * 4),
    "qdb_model_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "qdb_model_free": (None, [ctypes.c_void_p]),
    "qdb_model_set_mask_eos": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qdb_session_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int]),
    "qdb_session_free": (None, [ctypes.c_void_p]),
    "qdb_session_capacity": (ctypes.c_int, [ctypes.c_void_p]),
    "qdb_session_reserve": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qdb_prefill": (ctypes.c_int, [ctypes.c_void_p, _f32p, ctypes.c_int, ctypes.c_int]),
    "qdb_prefill_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int]),
    "qdb_prefill_batch": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _f32p, _i32p, _i32p]),
    "qdb_prefill_batch_device": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, ctypes.c_void_p,
                                                _i32p, _i32p]),
    "qdb_forward": (ctypes.c_int, [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, _f32p]),
    "qdb_decode_greedy": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p]),
    "qdb_forward_batch": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _f32p, _i32p, _i32p, _f32p]),
    "qdb_decode_greedy_batch": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _i32p, _i32p,
                                               ctypes.c_int, _i32p]),
    "qdb_model_sync": (ctypes.c_int, [ctypes.c_void_p]),
    "qdb_mel_frames": (ctypes.c_int, [ctypes.c_int]),
    "qdb_build_prompt_device": (ctypes.c_int, [ctypes.c_void_p, _i32p, ctypes.c_int, ctypes.c_void_p,
                                               ctypes.c_void_p]),
    "qdb_encoder_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int]),
    "qdb_encoder_free": (None, [ctypes.c_void_p]),
    "qdb_encoder_set_stem": (ctypes.c_int, [ctypes.c_void_p] + [_f32p] * 6 + [_u16p]),
    "qdb_encoder_set_layer": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int] + [_u16p, _f32p] * 4 + [_f32p, _f32p]
                              + [_u16p, _f32p] * 2 + [_f32p, _f32p]),
    "qdb_encoder_set_post": (ctypes.c_int, [ctypes.c_void_p, _f32p, _f32p, _u16p, _f32p, _u16p, _f32p]),
    "qdb_encoder_finalize": (ctypes.c_int, [ctypes.c_void_p]),
    "qdb_encoder_tokens": (ctypes.c_int, [ctypes.c_int]),
    "qdb_encoder_forward": (ctypes.POINTER(ctypes.c_float), [ctypes.c_void_p, _f32p, ctypes.c_int, _i32p]),
    "qdb_encoder_forward_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "qdb_encoder_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "qdb_encoder_forward_batch_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_void_p),
                                                        _i32p, ctypes.c_void_p]),
    "qdb_streams_create": (ctypes.c_void_p, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "qdb_streams_free": (None, [ctypes.c_void_p]),
    "qdb_streams_chunk": (ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_void_p), _i32p, _i32p, _i32p,
                                         _i32p]),
    "qdb_streams_tokens": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, _i32p, ctypes.c_int]),
    "qdb_streams_stats": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.POINTER(ctypes.c_longlong)]),
    "qdb_streams_reset": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    "qdb_streams_last_chunk": (ctypes.c_int, [ctypes.c_void_p, _f32p, _i32p]),
    "qdb_mel_spectrogram": (ctypes.POINTER(ctypes.c_float), [_f32p, ctypes.c_int, _i32p]),
    "qdb_mel_spectrogram_device": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]),
    "qdb_forward_noalloc": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]),
    "qdb_model_stream": (ctypes.c_void_p, [ctypes.c_void_p]),
    "qdb_model_set_wait_limit": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_longlong]),
    "qdb_trace_step": (ctypes.c_int, [ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                      ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]),
    "qdb_trace_batch_step": (ctypes.c_int, [ctypes.POINTER(ctypes.c_void_p), ctypes.c_int, _f32p, _i32p,
                                            ctypes.POINTER(ctypes.c_uint64), ctypes.c_int]),
}


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is missing: build it with `make -C qwen-asr_b200` "
                          "(the CUDA library is the only compute path)")
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in ABI.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    return lib


lib = _load()

# At interpreter exit the process releases device memory itself; finalizers
# then skip their frees (object finalization order is arbitrary at shutdown).
_exiting = [False]
atexit.register(lambda: _exiting.__setitem__(0, True))


class QdbError(RuntimeError):
    pass


def _err(what):
    msg = lib.qdb_last_error()
    return QdbError(f"{what}: {msg.decode() if msg else ''}")


def _ptr(a, t):
    return a.ctypes.data_as(t)


def device_count() -> int:
    return lib.qdb_device_count()


class Model:
    """Device copy of one decoder's weights (replaces qwen_decoder_load,
    qwen_asr_decoder.c:45-116). `weights` is a synth.WeightSet or any object
    with .cfg, .embed, .final_norm and .layer(i)."""

    def __init__(self, weights, device: int = 0, mask_eos: bool = False):
        cfg = weights.cfg
        self.cfg = cfg
        c = QdbConfig(cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.intermediate,
                      cfg.vocab, cfg.eps, cfg.theta)
        self.h = lib.qdb_model_create(ctypes.byref(c), device)
        if not self.h:
            raise _err("qdb_model_create")
        emb = np.ascontiguousarray(weights.embed)
        fn = np.ascontiguousarray(weights.final_norm, dtype=np.float32)
        if lib.qdb_model_set_embed(self.h, _ptr(emb, _u16p), _ptr(fn, _f32p)):
            raise _err("qdb_model_set_embed")
        for i in range(cfg.layers):
            L = weights.layer(i)
            mats = [np.ascontiguousarray(L[k]) for k in ("wq", "wk", "wv", "wo", "gate", "up", "down")]
            norms = [np.ascontiguousarray(L[k], dtype=np.float32)
                     for k in ("q_norm", "k_norm", "input_norm", "post_attn_norm")]
            if lib.qdb_model_set_layer(self.h, i, *[_ptr(a, _u16p) for a in mats], *[_ptr(a, _f32p) for a in norms]):
                raise _err(f"qdb_model_set_layer({i})")
        if lib.qdb_model_finalize(self.h):
            raise _err("qdb_model_finalize")
        self.set_mask_eos(mask_eos)

    def set_mask_eos(self, on: bool):
        lib.qdb_model_set_mask_eos(self.h, 1 if on else 0)

    def set_wait_limit(self, cycles: int):
        """Bound (SM cycles) on the kernels' data waits on this model's device;
        negative restores the default (about one second)."""
        if lib.qdb_model_set_wait_limit(self.h, int(cycles)):
            raise _err("qdb_model_set_wait_limit")

    @property
    def stream_handle(self) -> int:
        """cudaStream_t of this model (for torch.cuda.ExternalStream)."""
        return lib.qdb_model_stream(self.h) or 0

    def build_prompt_device(self, desc, audio_ptr: int, out_ptr: int):
        """Prompt rows on the device: desc[r] >= 0 token id, < 0 audio row -(desc[r]+1)
        of audio_ptr [*, hidden]; out_ptr [len(desc), hidden] f32 (model's stream)."""
        d = np.ascontiguousarray(desc, dtype=np.int32)
        if lib.qdb_build_prompt_device(self.h, _ptr(d, _i32p), len(d), ctypes.c_void_p(audio_ptr),
                                       ctypes.c_void_p(out_ptr)):
            raise _err("qdb_build_prompt_device")

    def session(self, capacity: int = 1024) -> "Session":
        return Session(self, capacity)

    def sync(self):
        if lib.qdb_model_sync(self.h):
            raise _err("qdb_model_sync")

    def close(self):
        if self.h and not _exiting[0]:
            lib.qdb_model_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """One utterance's device KV cache (qwen_ctx_t KV fields)."""

    def __init__(self, model: Model, capacity: int = 1024):
        self.model = model
        self.h = lib.qdb_session_create(model.h, capacity)
        if not self.h:
            raise _err("qdb_session_create")

    @property
    def capacity(self) -> int:
        return lib.qdb_session_capacity(self.h)

    def prefill(self, embeds: np.ndarray, start_pos: int):
        e = np.ascontiguousarray(embeds, dtype=np.float32)
        n = 0 if e.size == 0 else e.shape[0]
        if lib.qdb_prefill(self.h, _ptr(e, _f32p), n, start_pos):
            raise _err("qdb_prefill")

    def prefill_device(self, dev_ptr: int, n: int, start_pos: int):
        if lib.qdb_prefill_device(self.h, ctypes.c_void_p(dev_ptr), n, start_pos):
            raise _err("qdb_prefill_device")

    def forward(self, embed: np.ndarray, pos: int, want_hidden=False, want_logits=False):
        cfg = self.model.cfg
        e = np.ascontiguousarray(embed, dtype=np.float32).reshape(cfg.hidden)
        hid = np.empty(cfg.hidden, np.float32) if want_hidden else None
        log = np.empty(cfg.vocab, np.float32) if want_logits else None
        tok = lib.qdb_forward(self.h, _ptr(e, _f32p), pos, _ptr(hid, _f32p) if hid is not None else None,
                              _ptr(log, _f32p) if log is not None else None)
        if tok < 0:
            raise _err("qdb_forward")
        return tok, hid, log

    def decode_greedy(self, first_token: int, pos: int, n_steps: int) -> np.ndarray:
        out = np.empty(max(n_steps, 1), np.int32)
        if lib.qdb_decode_greedy(self.h, first_token, pos, n_steps, _ptr(out, _i32p)):
            raise _err("qdb_decode_greedy")
        return out[:n_steps]

    def trace_step(self, token: int, pos: int, max_ctas: int = 1024) -> np.ndarray:
        """One greedy step with per-phase globaltimer stamps: [ctas, events] ns."""
        L = self.model.cfg.layers
        ev = 1 + 9 * L + 3
        buf = np.zeros(max_ctas * ev, np.uint64)
        n = lib.qdb_trace_step(self.h, token, pos, buf.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), buf.size)
        if n < 0:
            raise _err("qdb_trace_step")
        t = buf.reshape(-1, ev)
        return t[t[:, 0] != 0]

    def close(self):
        if self.h and not _exiting[0]:
            lib.qdb_session_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _handles(sessions):
    arr = (ctypes.c_void_p * len(sessions))(*[s.h for s in sessions])
    return arr


def prefill_batch(sessions, embeds, start_pos, lens=None):
    """Prefill of several sessions as one row batch. embeds: a list of f32
    [n_i, hidden] arrays (one per session), or, with lens, one f32 array of
    all rows back to back. start_pos: first position of each session."""
    n = len(sessions)
    sp = np.ascontiguousarray(start_pos, dtype=np.int32)
    if lens is None:
        ln = np.array([0 if e is None else len(e) for e in embeds], np.int32)
        rows = [np.asarray(e, np.float32) for e in embeds if e is not None and len(e)]
        cat = np.ascontiguousarray(np.concatenate(rows, axis=0)) if rows else np.zeros((1, 1), np.float32)
    else:
        ln = np.ascontiguousarray(lens, dtype=np.int32)
        cat = np.ascontiguousarray(embeds, dtype=np.float32)
    if lib.qdb_prefill_batch(_handles(sessions), n, _ptr(cat, _f32p), _ptr(ln, _i32p), _ptr(sp, _i32p)):
        raise _err("qdb_prefill_batch")


def prefill_batch_device(sessions, dev_ptr: int, lens, start_pos):
    """prefill_batch with the rows already on the device (dev_ptr: f32
    [sum(lens), hidden])."""
    n = len(sessions)
    ln = np.ascontiguousarray(lens, dtype=np.int32)
    sp = np.ascontiguousarray(start_pos, dtype=np.int32)
    if lib.qdb_prefill_batch_device(_handles(sessions), n, ctypes.c_void_p(dev_ptr), _ptr(ln, _i32p),
                                    _ptr(sp, _i32p)):
        raise _err("qdb_prefill_batch_device")


def forward_batch(sessions, embeds: np.ndarray, pos, want_logits: bool = False):
    """One decode step of independent sessions; returns the tokens, or
    (tokens, logits [n, vocab]) with want_logits."""
    n = len(sessions)
    e = np.ascontiguousarray(embeds, dtype=np.float32)
    p = np.ascontiguousarray(pos, dtype=np.int32)
    out = np.empty(n, np.int32)
    log = np.empty((n, sessions[0].model.cfg.vocab), np.float32) if want_logits else None
    if lib.qdb_forward_batch(_handles(sessions), n, _ptr(e, _f32p), _ptr(p, _i32p), _ptr(out, _i32p),
                             _ptr(log, _f32p) if log is not None else None):
        raise _err("qdb_forward_batch")
    return (out, log) if want_logits else out


def trace_batch_step(sessions, embeds: np.ndarray, pos, max_ctas: int = 1024) -> np.ndarray:
    """One persistent batched step with per-phase globaltimer stamps: returns
    ([ctas, events], [ctas, 256] layer-1 detail) ns (include/qwen_asr_b200.h)."""
    n = len(sessions)
    L = sessions[0].model.cfg.layers
    ev = 8 * L + 3
    e = np.ascontiguousarray(embeds, dtype=np.float32)
    p = np.ascontiguousarray(pos, dtype=np.int32)
    buf = np.zeros(max_ctas * (ev + 256), np.uint64)
    k = lib.qdb_trace_batch_step(_handles(sessions), n, _ptr(e, _f32p), _ptr(p, _i32p),
                                 buf.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), buf.size)
    if k < 0:
        raise _err("qdb_trace_batch_step")
    t = buf[:max_ctas * ev].reshape(-1, ev)
    ctas = int((t[:, -1] != 0).sum())
    return t[:ctas], buf[ctas * ev:ctas * ev + ctas * 256].reshape(ctas, 256)


class QdbStreamConfig(ctypes.Structure):
    _fields_ = [("max_new_tokens", ctypes.c_int), ("rollback", ctypes.c_int), ("unfixed_chunks", ctypes.c_int),
                ("past_text", ctypes.c_int),
                ("head_tokens", _i32p), ("n_head_tokens", ctypes.c_int),
                ("tail_tokens", _i32p), ("n_tail_tokens", ctypes.c_int),
                ("suffix_tokens", _i32p), ("n_suffix_tokens", ctypes.c_int),
                ("prompt_tokens", _i32p), ("n_prompt_tokens", ctypes.c_int),
                ("force_tokens", _i32p), ("n_force_tokens", ctypes.c_int),
                ("asr_text_token", ctypes.c_int)]


class Streams:
    """Many concurrent streams of one model (qdb_streams_*): the decoder side of
    the reference's streaming mode (stream_impl, qwen_asr.c:1214-2152), one
    chunk of every stream per call. Token-template keys (head, tail, suffix,
    prompt, force) take id lists; None keeps the reference's ids."""

    def __init__(self, model: Model, n_streams: int, max_new_tokens=32, rollback=5, unfixed_chunks=2,
                 past_text=False, head=None, tail=None, suffix=None, prompt=None, force=None, asr_text_token=0):
        self.model = model
        self.n = n_streams
        c = QdbStreamConfig(max_new_tokens, rollback, unfixed_chunks, 1 if past_text else 0)
        self._keep = []
        for name, v in (("head", head), ("tail", tail), ("suffix", suffix), ("prompt", prompt), ("force", force)):
            if v is not None:
                a = np.ascontiguousarray(v, dtype=np.int32)
                self._keep.append(a)
                setattr(c, name + "_tokens", _ptr(a, _i32p))
                setattr(c, "n_" + name + "_tokens", len(a))
        c.asr_text_token = asr_text_token
        self.h = lib.qdb_streams_create(model.h, n_streams, ctypes.byref(c))
        if not self.h:
            raise _err("qdb_streams_create")

    def chunk(self, audio, is_final):
        """audio: list of float32 [rows, hidden] arrays (0 rows = no encoder
        output this chunk, None = stream not in this call); is_final: list of
        bools. Returns (n_emitted, reset) int arrays."""
        arrs = [None if a is None else np.ascontiguousarray(a, dtype=np.float32) for a in audio]
        ptrs = (ctypes.c_void_p * self.n)(*[a.ctypes.data if a is not None and a.size else None for a in arrs])
        lens = np.array([-1 if a is None else (a.shape[0] if a.size else 0) for a in arrs], np.int32)
        fin = np.ascontiguousarray(is_final, dtype=np.int32)
        ne = np.zeros(self.n, np.int32)
        rs = np.zeros(self.n, np.int32)
        if lib.qdb_streams_chunk(self.h, ptrs, _ptr(lens, _i32p), _ptr(fin, _i32p), _ptr(ne, _i32p),
                                 _ptr(rs, _i32p)):
            raise _err("qdb_streams_chunk")
        return ne, rs

    def tokens(self, i: int, which: str = "emitted") -> np.ndarray:
        w = {"emitted": 0, "raw": 1, "stable": 2}[which]
        n = lib.qdb_streams_tokens(self.h, i, w, None, 0)
        if n < 0:
            raise _err("qdb_streams_tokens")
        out = np.zeros(max(n, 1), np.int32)
        lib.qdb_streams_tokens(self.h, i, w, _ptr(out, _i32p), n)
        return out[:n]

    def stats(self, i: int) -> dict:
        v = (ctypes.c_longlong * 8)()
        if lib.qdb_streams_stats(self.h, i, v):
            raise _err("qdb_streams_stats")
        keys = ("chunk_idx", "chunks", "prefill_total", "prefill_reused", "decoded", "last_generated",
                "last_reused", "last_prefill_len")
        return dict(zip(keys, list(v)))

    def reset(self, i: int):
        """Restart stream i as a new stream (its KV storage is kept)."""
        if lib.qdb_streams_reset(self.h, i):
            raise _err("qdb_streams_reset")

    def last_chunk(self) -> dict:
        """Device ms of the last chunk's prefill and greedy loop, streams run, rows prefilled."""
        ms = np.zeros(2, np.float32)
        cnt = np.zeros(2, np.int32)
        lib.qdb_streams_last_chunk(self.h, _ptr(ms, _f32p), _ptr(cnt, _i32p))
        return {"prefill_ms": float(ms[0]), "decode_ms": float(ms[1]), "active": int(cnt[0]), "rows": int(cnt[1])}

    def close(self):
        if self.h and not _exiting[0]:
            lib.qdb_streams_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class QdbEncoderConfig(ctypes.Structure):
    _fields_ = [(k, ctypes.c_int) for k in ("d_model", "layers", "heads", "head_dim", "ffn_dim", "output_dim")]


class Encoder:
    """Device copy of the audio encoder (replaces qwen_encoder_load,
    qwen_asr_encoder.c:66-168). `weights` is a synth.EncoderWeightSet or any
    object with .cfg (d_model, layers, heads, head_dim, ffn, output_dim) and
    .view(name) / .f32(name) over the reference's tensor names."""

    def __init__(self, weights, device: int = 0):
        ec = weights.cfg
        self.cfg = ec
        c = QdbEncoderConfig(ec.d_model, ec.layers, ec.heads, ec.head_dim, ec.ffn, ec.output_dim)
        self.h = lib.qdb_encoder_create(ctypes.byref(c), device)
        if not self.h:
            raise _err("qdb_encoder_create")
        p = "thinker.audio_tower."
        f = lambda n: np.ascontiguousarray(weights.f32(p + n), dtype=np.float32)
        u = lambda n: np.ascontiguousarray(weights.view(p + n))
        stem = [f("conv2d1.weight"), f("conv2d1.bias"), f("conv2d2.weight"), f("conv2d2.bias"),
                f("conv2d3.weight"), f("conv2d3.bias")]
        cout = u("conv_out.weight")
        if lib.qdb_encoder_set_stem(self.h, *[_ptr(a, _f32p) for a in stem], _ptr(cout, _u16p)):
            raise _err("qdb_encoder_set_stem")
        for i in range(ec.layers):
            q = f"layers.{i}."
            args = []
            for nm in ("q_proj", "k_proj", "v_proj", "out_proj"):
                args += [u(q + f"self_attn.{nm}.weight"), f(q + f"self_attn.{nm}.bias")]
            args += [f(q + "self_attn_layer_norm.weight"), f(q + "self_attn_layer_norm.bias")]
            args += [u(q + "fc1.weight"), f(q + "fc1.bias"), u(q + "fc2.weight"), f(q + "fc2.bias")]
            args += [f(q + "final_layer_norm.weight"), f(q + "final_layer_norm.bias")]
            ptrs = [_ptr(a, _u16p if a.dtype == np.uint16 else _f32p) for a in args]
            if lib.qdb_encoder_set_layer(self.h, i, *ptrs):
                raise _err(f"qdb_encoder_set_layer({i})")
        post = [f("ln_post.weight"), f("ln_post.bias"), u("proj1.weight"), f("proj1.bias"), u("proj2.weight"),
                f("proj2.bias")]
        if lib.qdb_encoder_set_post(self.h, *[_ptr(a, _u16p if a.dtype == np.uint16 else _f32p) for a in post]):
            raise _err("qdb_encoder_set_post")
        if lib.qdb_encoder_finalize(self.h):
            raise _err("qdb_encoder_finalize")

    @staticmethod
    def tokens(mel_frames: int) -> int:
        return lib.qdb_encoder_tokens(int(mel_frames))

    def forward(self, mel: np.ndarray) -> np.ndarray:
        """Mirror of qwen_encoder_forward: mel [128, frames] -> [tokens, output_dim]."""
        m = np.ascontiguousarray(mel, dtype=np.float32)
        n = ctypes.c_int(0)
        p = lib.qdb_encoder_forward(self.h, _ptr(m, _f32p), m.shape[1], ctypes.byref(n))
        if not p:
            raise _err("qdb_encoder_forward")
        try:
            return np.ctypeslib.as_array(p, (n.value, self.cfg.output_dim)).copy()
        finally:
            _libc.free(ctypes.cast(p, ctypes.c_void_p))

    def forward_device(self, mel_ptr: int, frames: int, out_ptr: int) -> int:
        """Device form on the encoder's stream; returns the token count."""
        n = lib.qdb_encoder_forward_device(self.h, ctypes.c_void_p(mel_ptr), int(frames), ctypes.c_void_p(out_ptr))
        if n < 0:
            raise _err("qdb_encoder_forward_device")
        return n

    def forward_batch_device(self, mel_ptrs, frames, out_ptr: int) -> int:
        """Many utterances in one pass (device pointers); returns the total token count."""
        n = len(mel_ptrs)
        ptrs = (ctypes.c_void_p * n)(*mel_ptrs)
        f = np.ascontiguousarray(frames, dtype=np.int32)
        r = lib.qdb_encoder_forward_batch_device(self.h, n, ptrs, _ptr(f, _i32p), ctypes.c_void_p(out_ptr))
        if r < 0:
            raise _err("qdb_encoder_forward_batch_device")
        return r

    @property
    def stream_handle(self) -> int:
        return lib.qdb_encoder_stream(self.h) or 0

    def close(self):
        if self.h and not _exiting[0]:
            lib.qdb_encoder_free(self.h)
        self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


_libc = ctypes.CDLL(None)
_libc.free.argtypes = [ctypes.c_void_p]
_libc.free.restype = None


def mel_frames(n_samples: int) -> int:
    """Frames the log-mel of n_samples has (<= 0: too short)."""
    return lib.qdb_mel_frames(int(n_samples))


def mel_spectrogram(samples: np.ndarray):
    """Mirror of qwen_mel_spectrogram (qwen_asr_audio.c:293): 16 kHz mono
    samples -> float32 [128, n_frames] computed on the current CUDA device, or
    None when the audio is too short (the reference returns NULL). Other
    failures raise."""
    x = np.ascontiguousarray(samples, dtype=np.float32)
    nf = ctypes.c_int(0)
    p = lib.qdb_mel_spectrogram(_ptr(x, _f32p), len(x), ctypes.byref(nf))
    if not p:
        if mel_frames(len(x)) <= 0:
            return None
        raise _err("qdb_mel_spectrogram")
    try:
        return np.ctypeslib.as_array(p, (128, nf.value)).copy()
    finally:
        _libc.free(ctypes.cast(p, ctypes.c_void_p))


def mel_spectrogram_device(samples_ptr: int, n_samples: int, mel_ptr: int, stream: int = 0) -> None:
    """Device form: float32 samples at samples_ptr -> float32 [128, mel_frames(n)]
    at mel_ptr, enqueued on `stream` (a cudaStream_t handle, 0 = default)."""
    if lib.qdb_mel_spectrogram_device(ctypes.c_void_p(samples_ptr), int(n_samples), ctypes.c_void_p(mel_ptr),
                                      ctypes.c_void_p(stream)):
        raise _err("qdb_mel_spectrogram_device")


def decode_greedy_batch(sessions, first_tokens, pos, n_steps: int) -> np.ndarray:
    n = len(sessions)
    f = np.ascontiguousarray(first_tokens, dtype=np.int32)
    p = np.ascontiguousarray(pos, dtype=np.int32)
    out = np.empty((max(n_steps, 1), n), np.int32)
    if lib.qdb_decode_greedy_batch(_handles(sessions), n, _ptr(f, _i32p), _ptr(p, _i32p), n_steps,
                                   _ptr(out, _i32p)):
        raise _err("qdb_decode_greedy_batch")
    return out[:n_steps]


class Decoder:
    """Mirror of the reference's per-context decoder calls. kv_cache_len is
    host-owned exactly like qwen_ctx_t.kv_cache_len (the caller may reset or
    rewind it, qwen_asr.c:704, :1764). Errors follow the reference: prefill
    returns silently leaving kv_cache_len unchanged (qwen_asr_decoder.c:276-282)
    and forward returns QWEN_TOKEN_IM_END (qwen_asr_decoder.c:417, :421); the
    message is kept in .last_error."""

    def __init__(self, model: Model, capacity: int = 1024):
        self.session = Session(model, capacity)
        self.kv_cache_len = 0
        self.dec_x = None  # final-normed hidden of the last forward (ctx->dec_x)
        self.last_error = ""

    def prefill(self, input_embeds: np.ndarray, seq_len: int | None = None):
        e = np.asarray(input_embeds, dtype=np.float32)
        if seq_len is None:
            seq_len = e.shape[0]
        try:
            self.session.prefill(e[:seq_len], self.kv_cache_len)
        except QdbError as ex:
            self.last_error = str(ex)
            return
        self.kv_cache_len += seq_len

    def forward(self, input_embed: np.ndarray, want_logits: bool = False):
        try:
            tok, hid, log = self.session.forward(input_embed, self.kv_cache_len, want_hidden=True,
                                                 want_logits=want_logits)
        except QdbError as ex:
            self.last_error = str(ex)
            return QWEN_TOKEN_IM_END
        self.kv_cache_len += 1
        self.dec_x = hid
        self.logits = log
        return tok
