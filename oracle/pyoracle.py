"""ctypes bindings of the CPU checkers. TEST INFRASTRUCTURE ONLY.

* Oracle  - liboracle.so, the C restatement of the reference decoder
            (qdec_oracle.c).
* RefDecoder - oracle/_ref/<isa>/libqwen_ref.so, the reference's own decoder
            sources compiled unmodified and driven by ref_harness.c.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline / reference
arm may use this module.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")

_f32p = ctypes.POINTER(ctypes.c_float)
_u16p = ctypes.POINTER(ctypes.c_uint16)
_i32p = ctypes.POINTER(ctypes.c_int)


class OrcConfig(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int), ("layers", ctypes.c_int), ("heads", ctypes.c_int),
                ("kv_heads", ctypes.c_int), ("head_dim", ctypes.c_int), ("intermediate", ctypes.c_int),
                ("vocab", ctypes.c_int), ("eps", ctypes.c_float), ("theta", ctypes.c_float)]


def _p(a, t):
    return a.ctypes.data_as(t)


def host_cpu_flags() -> set:
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("flags"):
                    return set(line.split(":", 1)[1].split())
    except OSError:
        pass
    return set()


def ref_so_path() -> str | None:
    """AVX-512 build when the host CPU has it, else the AVX2 build."""
    flags = host_cpu_flags()
    isa = "v4" if {"avx512f", "avx512bw", "avx512vl", "avx512dq"} <= flags else "v3"
    p = os.path.join(HERE, "_ref", isa, "libqwen_ref.so")
    return p if os.path.exists(p) else None


_orc = None


def _oracle_lib():
    global _orc
    if _orc is None:
        lib = ctypes.CDLL(ORACLE_SO)
        lib.orc_model_create.restype = ctypes.c_void_p
        lib.orc_model_create.argtypes = [ctypes.POINTER(OrcConfig), _u16p, _f32p]
        lib.orc_model_set_layer.restype = ctypes.c_int
        lib.orc_model_set_layer.argtypes = [ctypes.c_void_p, ctypes.c_int] + [_u16p] * 7 + [_f32p] * 4
        lib.orc_model_free.argtypes = [ctypes.c_void_p]
        lib.orc_state_create.restype = ctypes.c_void_p
        lib.orc_state_create.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.orc_state_free.argtypes = [ctypes.c_void_p]
        lib.orc_state_len.restype = ctypes.c_int
        lib.orc_state_len.argtypes = [ctypes.c_void_p]
        lib.orc_state_set_len.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.orc_state_set_kv_round.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.orc_prefill.restype = ctypes.c_int
        lib.orc_prefill.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int]
        lib.orc_forward.restype = ctypes.c_int
        lib.orc_forward.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, _f32p]
        lib.orc_matvec_bf16.argtypes = [_f32p, _f32p, _u16p, ctypes.c_int, ctypes.c_int]
        lib.orc_argmax_matvec_bf16.restype = ctypes.c_int
        lib.orc_argmax_matvec_bf16.argtypes = [_f32p, _u16p, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        lib.orc_rms_norm.argtypes = [_f32p, _f32p, _f32p, ctypes.c_int, ctypes.c_int, ctypes.c_float]
        lib.orc_set_threads.argtypes = [ctypes.c_int]
        _orc = lib
    return _orc


class Oracle:
    """The C restatement over a synth.WeightSet (weights are borrowed)."""

    def __init__(self, ws, max_pos: int = 2048, threads: int | None = None):
        self.lib = _oracle_lib()
        self.lib.orc_set_threads(threads or os.cpu_count() or 1)
        self.ws = ws
        cfg = ws.cfg
        self.cfg = cfg
        self._keep = []
        c = OrcConfig(*cfg.as_tuple(), cfg.eps, cfg.theta)
        fn = np.ascontiguousarray(ws.final_norm, dtype=np.float32)
        self._keep.append(fn)
        self.m = self.lib.orc_model_create(ctypes.byref(c), _p(ws.embed, _u16p), _p(fn, _f32p))
        for i in range(cfg.layers):
            L = ws.layer(i)
            mats = [L[k] for k in ("wq", "wk", "wv", "wo", "gate", "up", "down")]
            norms = [np.ascontiguousarray(L[k], dtype=np.float32)
                     for k in ("q_norm", "k_norm", "input_norm", "post_attn_norm")]
            self._keep += norms
            self.lib.orc_model_set_layer(self.m, i, *[_p(a, _u16p) for a in mats], *[_p(a, _f32p) for a in norms])
        self.s = self.lib.orc_state_create(self.m, max_pos)

    @property
    def kv_cache_len(self):
        return self.lib.orc_state_len(self.s)

    @kv_cache_len.setter
    def kv_cache_len(self, v):
        self.lib.orc_state_set_len(self.s, v)

    def set_kv_round(self, mode: int):
        self.lib.orc_state_set_kv_round(self.s, mode)

    def prefill(self, embeds):
        e = np.ascontiguousarray(embeds, dtype=np.float32)
        if e.shape[0] and self.lib.orc_prefill(self.s, _p(e, _f32p), e.shape[0]):
            raise RuntimeError("oracle prefill: capacity exceeded")

    def forward(self, embed, mask_eos=False, want_logits=True):
        e = np.ascontiguousarray(embed, dtype=np.float32)
        log = np.empty(self.cfg.vocab, np.float32) if want_logits else None
        hid = np.empty(self.cfg.hidden, np.float32)
        tok = self.lib.orc_forward(self.s, _p(e, _f32p), 1 if mask_eos else 0,
                                   _p(log, _f32p) if log is not None else None, _p(hid, _f32p))
        return tok, hid, log

    def close(self):
        if self.s:
            self.lib.orc_state_free(self.s)
            self.lib.orc_model_free(self.m)
            self.s = self.m = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class RefDecoder:
    """The reference's own qwen_decoder_load / prefill / forward (unmodified
    sources in oracle/_ref) over the same weight blob."""

    def __init__(self, ws, threads: int = 1, so_path: str | None = None):
        path = so_path or ref_so_path()
        if not path:
            raise FileNotFoundError("oracle/_ref not built (run `make -C oracle ref` where the reference tree exists)")
        lib = ctypes.CDLL(path)
        lib.refh_create.restype = ctypes.c_void_p
        lib.refh_create.argtypes = [_i32p, ctypes.c_float, ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
                                    ctypes.c_char_p, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                                    _i32p, _i32p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
        lib.refh_len.restype = ctypes.c_int
        lib.refh_len.argtypes = [ctypes.c_void_p]
        lib.refh_set_len.argtypes = [ctypes.c_void_p, ctypes.c_int]
        lib.refh_prefill.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int]
        lib.refh_forward.restype = ctypes.c_int
        lib.refh_forward.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, _f32p]
        lib.refh_decode_loop.restype = ctypes.c_double
        lib.refh_decode_loop.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, _i32p]
        lib.refh_now_ms.restype = ctypes.c_double
        lib.refh_free.argtypes = [ctypes.c_void_p]
        self.lib = lib
        self.path = path
        self.ws = ws
        self.cfg = cfg = ws.cfg
        names, offs, sizes, shapes = ws.table()
        n = len(names)
        cfg_arr = np.array(cfg.as_tuple(), dtype=np.int32)
        name_blob = b"".join(nm.encode() + b"\0" for nm in names)
        offs_a = np.array(offs, dtype=np.int64)
        sizes_a = np.array(sizes, dtype=np.int64)
        dt = np.full(n, 2, dtype=np.int32)  # DTYPE_BF16
        nd = np.array([2 if s[1] else 1 for s in shapes], dtype=np.int32)
        sh = np.array(shapes, dtype=np.int64).reshape(-1)
        self._keep = (cfg_arr, name_blob, offs_a, sizes_a, dt, nd, sh)
        self.h = lib.refh_create(_p(cfg_arr, _i32p), cfg.eps, cfg.theta, ctypes.c_void_p(ws.blob.ctypes.data), n,
                                 name_blob, _p(offs_a, ctypes.POINTER(ctypes.c_int64)),
                                 _p(sizes_a, ctypes.POINTER(ctypes.c_int64)), _p(dt, _i32p), _p(nd, _i32p),
                                 _p(sh, ctypes.POINTER(ctypes.c_int64)), threads)
        if not self.h:
            raise RuntimeError("reference qwen_decoder_load failed")

    @property
    def kv_cache_len(self):
        return self.lib.refh_len(self.h)

    @kv_cache_len.setter
    def kv_cache_len(self, v):
        self.lib.refh_set_len(self.h, v)

    def prefill(self, embeds):
        e = np.ascontiguousarray(embeds, dtype=np.float32)
        self.lib.refh_prefill(self.h, _p(e, _f32p), e.shape[0])

    def forward(self, embed, mask_eos=False, want_logits=True):
        e = np.ascontiguousarray(embed, dtype=np.float32)
        log = np.empty(self.cfg.vocab, np.float32) if want_logits else None
        hid = np.empty(self.cfg.hidden, np.float32)
        tok = self.lib.refh_forward(self.h, _p(e, _f32p), 1 if mask_eos else 0,
                                    _p(log, _f32p) if log is not None else None, _p(hid, _f32p))
        return tok, hid, log

    def decode_loop(self, first_token, n_steps, mask_eos=True):
        out = np.empty(n_steps, np.int32)
        ms = self.lib.refh_decode_loop(self.h, first_token, n_steps, 1 if mask_eos else 0, _p(out, _i32p))
        return out, ms

    def now_ms(self):
        return self.lib.refh_now_ms()

    def close(self):
        if self.h:
            self.lib.refh_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def margin_top2(logits: np.ndarray, mask_eos: bool = False) -> float:
    l = logits.astype(np.float64).copy()
    if mask_eos and l.shape[0] > 151645:
        l[151643] = -np.inf
        l[151645] = -np.inf
    top = np.partition(l, -2)[-2:]
    return float(top[1] - top[0])


def ref_mel_spectrogram(samples, so_path: str | None = None):
    """The reference's own qwen_mel_spectrogram (qwen_asr_audio.c:293, compiled
    unmodified into oracle/_ref): [128, n_frames] float32, or None when it
    returns NULL (audio too short)."""
    path = so_path or ref_so_path()
    if not path:
        raise FileNotFoundError("oracle/_ref not built (run `make -C oracle ref` where the reference tree exists)")
    lib = ctypes.CDLL(path)
    lib.qwen_mel_spectrogram.restype = ctypes.POINTER(ctypes.c_float)
    lib.qwen_mel_spectrogram.argtypes = [_f32p, ctypes.c_int, _i32p]
    x = np.ascontiguousarray(samples, dtype=np.float32)
    nf = ctypes.c_int(0)
    p = lib.qwen_mel_spectrogram(_p(x, _f32p), len(x), ctypes.byref(nf))
    if not p:
        return None
    out = np.ctypeslib.as_array(p, (128, nf.value)).copy()
    libc = ctypes.CDLL(None)
    libc.free.argtypes = [ctypes.c_void_p]
    libc.free(ctypes.cast(p, ctypes.c_void_p))
    return out


class RefEncoder:
    """The reference's own qwen_encoder_load / qwen_encoder_forward
    (qwen_asr_encoder.c, compiled unmodified into oracle/_ref) over a
    synth.EncoderWeightSet blob."""

    def __init__(self, ews, threads: int = 1, so_path: str | None = None):
        path = so_path or ref_so_path()
        if not path:
            raise FileNotFoundError("oracle/_ref not built (run `make -C oracle ref` where the reference tree exists)")
        lib = ctypes.CDLL(path)
        lib.refh_encoder_create.restype = ctypes.c_void_p
        lib.refh_encoder_create.argtypes = [_i32p, ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p,
                                            ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64),
                                            _i32p, _i32p, ctypes.POINTER(ctypes.c_int64), ctypes.c_int]
        lib.refh_encoder_forward.restype = ctypes.c_int
        lib.refh_encoder_forward.argtypes = [ctypes.c_void_p, _f32p, ctypes.c_int, _f32p, ctypes.c_int]
        lib.refh_encoder_free.argtypes = [ctypes.c_void_p]
        self.lib, self.ews, self.cfg = lib, ews, ews.cfg
        names, offs, sizes, shapes = ews.table()
        n = len(names)
        ecfg = np.array(ews.cfg.as_tuple(), dtype=np.int32)
        name_blob = b"".join(nm.encode() + b"\0" for nm in names)
        offs_a = np.array(offs, dtype=np.int64)
        sizes_a = np.array(sizes, dtype=np.int64)
        dt = np.full(n, 2, dtype=np.int32)  # DTYPE_BF16
        nd = np.array([2 if s[1] else 1 for s in shapes], dtype=np.int32)
        sh = np.array(shapes, dtype=np.int64).reshape(-1)
        self._keep = (ecfg, name_blob, offs_a, sizes_a, dt, nd, sh)
        self.h = lib.refh_encoder_create(_p(ecfg, _i32p), ctypes.c_void_p(ews.blob.ctypes.data), n, name_blob,
                                         _p(offs_a, ctypes.POINTER(ctypes.c_int64)),
                                         _p(sizes_a, ctypes.POINTER(ctypes.c_int64)), _p(dt, _i32p), _p(nd, _i32p),
                                         _p(sh, ctypes.POINTER(ctypes.c_int64)), threads)
        if not self.h:
            raise RuntimeError("reference qwen_encoder_load failed")

    def forward(self, mel):
        """mel f32 [128, frames] -> f32 [seq, output_dim]"""
        mel = np.ascontiguousarray(mel, dtype=np.float32)
        frames = mel.shape[1]
        cap = frames  # seq <= frames
        out = np.empty((cap, self.cfg.output_dim), np.float32)
        n = self.lib.refh_encoder_forward(self.h, _p(mel, _f32p), frames, _p(out, _f32p), cap)
        if n < 0:
            raise RuntimeError("reference qwen_encoder_forward failed")
        return out[:n].copy()

    def close(self):
        if self.h:
            self.lib.refh_encoder_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
