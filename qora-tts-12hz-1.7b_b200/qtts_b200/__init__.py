"""Python mirror of the QORA-TTS decode-loop API over libqtts_b200.so.

The functions keep the names, argument meaning and error behaviour of the
reference crate's public functions (the Rust signatures are cited on each);
a ``Session`` plays the role of the reference's ``RawKvCache`` (the KV cache
lives on the GPU).  All compute runs in the sm_100a kernels of
libqtts_b200.so; this module only marshals host buffers.  There is no CPU
fallback: if the library is missing, importing this module raises.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
PKG_DIR = os.path.dirname(HERE)
LIB_PATH = os.path.join(PKG_DIR, "libqtts_b200.so")
HEADER = os.path.join(os.path.dirname(PKG_DIR), "include", "qtts.h")

OK = 0
ERR_BADARG, ERR_OOM, ERR_CUDA, ERR_TIMEOUT, ERR_FORMAT, ERR_IO, ERR_STATE, ERR_NODEV, ERR_RANGE = (
    -1, -2, -3, -4, -5, -6, -7, -8, -9)
IGNORE_EOS = 1
FULL_PROMPT = 2  # benchmark mode: the whole text prefilled (qtts.h QTTS_FULL_PROMPT)
SESSION_KV_F16 = 1  # opt-in f16 K/V caches (qtts.h QTTS_SESSION_KV_F16)
# kernel families of the frame plan (qtts.h QTTS_FAMILY_*)
FAMILY_Q4MV_DEC, FAMILY_Q4MV_ROWS, FAMILY_TC_PROJ, FAMILY_ATTN, FAMILY_Q4MV_BATCH = 1, 2, 3, 4, 5


class QttsError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"qtts error {code}: {msg}")
        self.code = code


class Dims(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "t_layers", "t_hidden", "t_text_hidden", "t_heads", "t_kv_heads", "t_head_dim",
        "t_inter", "t_vocab", "t_text_vocab", "t_max_pos")] + [("t_sec", C.c_int * 3)] + [
        (n, C.c_int) for n in ("p_layers", "p_hidden", "p_heads", "p_kv_heads", "p_head_dim",
                               "p_inter", "p_vocab", "p_groups", "p_max_pos", "fmt")]

    def as_dict(self):
        d = {n: getattr(self, n) for n, _ in self._fields_ if n != "t_sec"}
        d["t_sec"] = list(self.t_sec)
        return d


class SampleParams(C.Structure):
    """generate_new.rs:38-45 TTSParams (max_codes is an argument of generate)."""
    _fields_ = [("temperature", C.c_float), ("top_k", C.c_int),
                ("repetition_penalty", C.c_float), ("codec_eos_id", C.c_uint32)]


class Utterance(C.Structure):
    _fields_ = [("text", C.POINTER(C.c_uint32)), ("n_text", C.c_int), ("speaker_id", C.c_uint32),
                ("language_id", C.c_uint32), ("voice", C.POINTER(C.c_float)), ("seed", C.c_uint64),
                ("params", SampleParams)]


def _load():
    if not os.path.exists(LIB_PATH):
        raise ImportError(f"{LIB_PATH} is not built: run `make -C {PKG_DIR}` (the CUDA path has no fallback)")
    L = C.CDLL(LIB_PATH)
    P = C.c_void_p
    fp = C.POINTER(C.c_float)
    u32p = C.POINTER(C.c_uint32)
    sig = {
        "qtts_last_error": (C.c_char_p, []),
        "qtts_version": (C.c_int, []),
        "qtts_file_probe": (C.c_int, [C.c_char_p, C.POINTER(Dims)]),
        "qtts_synth_write": (C.c_int, [C.c_char_p, C.POINTER(Dims), C.c_uint64]),
        "qtts_synth_write_ex": (C.c_int, [C.c_char_p, C.POINTER(Dims), C.c_uint64, C.c_uint]),
        "qtts_decoder_load": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(P)]),
        "qtts_decoder_free": (C.c_int, [P]),
        "qtts_decoder_stream": (P, [P]),
        "qtts_decode_latent": (C.c_int, [P, C.POINTER(C.c_uint32), C.c_int, C.POINTER(C.c_float)]),
        "qtts_decode_latent_dev": (C.c_int, [P, P, C.c_int, P]),
        "qtts_decoder_sync": (C.c_int, [P]),
        "qtts_dims_1p7b": (None, [C.POINTER(Dims)]),
        "qtts_dims_tiny": (None, [C.POINTER(Dims)]),
        "qtts_model_load": (C.c_int, [C.c_char_p, C.c_int, C.POINTER(P)]),
        "qtts_model_free": (C.c_int, [P]),
        "qtts_model_dims": (C.c_int, [P, C.POINTER(Dims)]),
        "qtts_model_device_bytes": (C.c_size_t, [P]),
        "qtts_session_create": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(P)]),
        "qtts_session_create_ex": (C.c_int, [P, C.c_int, C.c_int, C.c_uint, C.POINTER(P)]),
        "qtts_session_free": (C.c_int, [P]),
        "qtts_session_reset": (C.c_int, [P]),
        "qtts_session_stream": (P, [P]),
        "qtts_session_set_wait_budget": (C.c_int, [P, C.c_uint64]),
        "qtts_embed_text": (C.c_int, [P, C.c_uint32, fp]),
        "qtts_embed_codec": (C.c_int, [P, C.c_uint32, fp]),
        "qtts_prefill": (C.c_int, [P, fp, C.c_int, fp, fp]),
        "qtts_talker_step": (C.c_int, [P, fp, C.c_int, fp]),
        "qtts_predict_acoustic": (C.c_int, [P, fp, fp, u32p]),
        "qtts_acoustic_embed_sum": (C.c_int, [P, u32p, fp]),
        "qtts_sample": (C.c_int, [P, fp, C.c_int, C.POINTER(SampleParams), u32p, C.POINTER(C.c_uint64), u32p]),
        "qtts_generate": (C.c_int, [P, C.c_int, C.POINTER(Utterance), C.c_int, C.c_uint, u32p, u32p,
                                    C.POINTER(C.c_int), fp, fp]),
        "qtts_generate_begin": (C.c_int, [P, C.c_int, C.POINTER(Utterance), C.c_int, C.c_uint, u32p]),
        "qtts_generate_frames": (C.c_int, [P, C.c_int]),
        "qtts_generate_end": (C.c_int, [P, u32p, C.POINTER(C.c_int), fp, fp]),
        "qtts_frame_kernel_count": (C.c_int, [P]),
        "qtts_frame_graph_captures": (C.c_int, [P]),
        "qtts_frame_family_time": (C.c_int, [P, C.c_int, C.c_int, C.POINTER(C.c_float), C.POINTER(C.c_int),
                                             C.POINTER(C.c_double), C.POINTER(C.c_double)]),
        "qtts_q4_gemv_scratch_bytes": (C.c_size_t, [C.c_int, C.c_int, C.c_int]),
        "qtts_q4_gemv_dev": (C.c_int, [P, P, C.c_int, C.c_int, P, C.c_int, P, P, C.c_size_t, P]),
        "qtts_q4_gemv": (C.c_int, [C.POINTER(C.c_uint8), C.POINTER(C.c_uint16), C.c_int, C.c_int, fp,
                                   C.c_int, fp]),
        "qtts_f16_gemv_dev": (C.c_int, [P, C.c_int, C.c_int, P, C.c_int, P, P]),
        "qtts_q4_dequant_dev": (C.c_int, [P, P, C.c_int, C.c_int, P, P]),
        "qtts_expf_dev": (C.c_int, [P, P, C.c_int, P]),
        "qtts_q4_quantize_dev": (C.c_int, [P, C.c_int, C.c_int, P, P, P]),
        "qtts_q4_quantize": (C.c_int, [fp, C.c_int, C.c_int, C.POINTER(C.c_uint8), C.POINTER(C.c_uint16)]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args
    return L


lib = _load()


def _check(rc: int):
    if rc != OK:
        raise QttsError(rc, lib.qtts_last_error().decode(errors="replace"))


def _fp(a):
    return a.ctypes.data_as(C.POINTER(C.c_float))


def _u32p(a):
    return a.ctypes.data_as(C.POINTER(C.c_uint32))


def dims_1p7b() -> Dims:
    d = Dims()
    lib.qtts_dims_1p7b(C.byref(d))
    return d


def dims_tiny() -> Dims:
    d = Dims()
    lib.qtts_dims_tiny(C.byref(d))
    return d


def synth_write(path: str, dims: Dims, seed: int = 0) -> None:
    """Seeded synthetic model in the save.rs layout (save.rs:23-137)."""
    _check(lib.qtts_synth_write(path.encode(), C.byref(dims), seed))


SYNTH_DECODER = 1  # qtts.h QTTS_SYNTH_DECODER


def synth_write_with_decoder(path: str, dims: Dims, seed: int = 0) -> None:
    """The synthetic model with a full-size speech decoder section
    (qtts.h qtts_synth_write_ex / QTTS_SYNTH_DECODER)."""
    _check(lib.qtts_synth_write_ex(path.encode(), C.byref(dims), seed, SYNTH_DECODER))


class Decoder:
    """The speech decoder's first stage on the GPU (decoder.rs:142-335 with
    the conv.rs:114-191 pre-conv): 16 code streams of T frames -> the
    transformer output [1024][T] (qtts.h qtts_decode_latent)."""

    def __init__(self, path: str, device: int = 0):
        h = C.c_void_p()
        _check(lib.qtts_decoder_load(path.encode(), device, C.byref(h)))
        self.h = h

    @property
    def stream(self) -> int:
        return lib.qtts_decoder_stream(self.h) or 0

    def decode_latent(self, codes) -> np.ndarray:
        codes = np.ascontiguousarray(codes, dtype=np.uint32)
        if codes.ndim != 2 or codes.shape[0] != 16:
            raise QttsError(ERR_BADARG, f"codes must be [16][T], got {codes.shape}")
        T = codes.shape[1]
        out = np.empty((1024, T), np.float32)
        _check(lib.qtts_decode_latent(self.h, codes.ctypes.data_as(C.POINTER(C.c_uint32)), T,
                                      out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def decode_latent_dev(self, codes_ptr: int, n_frames: int, out_ptr: int) -> None:
        """Device buffers (codes [16][T] u32, out [1024][T] f32), async on
        the decoder's stream; errors of the launch itself only."""
        _check(lib.qtts_decode_latent_dev(self.h, C.c_void_p(codes_ptr), n_frames, C.c_void_p(out_ptr)))

    def sync(self) -> None:
        _check(lib.qtts_decoder_sync(self.h))

    def close(self):
        if getattr(self, "h", None) and lib is not None:  # (lib is None at interpreter exit)
            lib.qtts_decoder_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def file_probe(path: str) -> Dims:
    """Parse + validate a .qora-tts file (save.rs:262-409) without a GPU."""
    d = Dims()
    _check(lib.qtts_file_probe(path.encode(), C.byref(d)))
    return d


class Model:
    """save::load_model (save.rs:262) uploaded to one GPU."""

    def __init__(self, path: str, device: int = 0):
        h = C.c_void_p()
        _check(lib.qtts_model_load(path.encode(), device, C.byref(h)))
        self.h = h
        self.dims = Dims()
        _check(lib.qtts_model_dims(self.h, C.byref(self.dims)))
        self.device_bytes = lib.qtts_model_device_bytes(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib.qtts_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Session:
    """The device KV caches of gemv.rs:77-86 (RawKvCache) for up to
    max_batch utterances of up to max_positions positions each."""

    def __init__(self, model: Model, max_batch: int = 1, max_positions: int = 2048, kv_f16: bool = False):
        """kv_f16: the opt-in f16 K/V caches (qtts.h QTTS_SESSION_KV_F16);
        the default is the reference's f32."""
        h = C.c_void_p()
        flags = SESSION_KV_F16 if kv_f16 else 0
        _check(lib.qtts_session_create_ex(model.h, max_batch, max_positions, flags, C.byref(h)))
        self.h = h
        self.model = model
        self.dims = model.dims
        self.H = model.dims.t_hidden
        self.V = model.dims.t_vocab

    @property
    def stream(self) -> int:
        return lib.qtts_session_stream(self.h) or 0

    def reset(self):
        _check(lib.qtts_session_reset(self.h))

    def set_wait_budget(self, ns: int):
        """Bound (ns) on the first device wait of each exchange in the one-row
        layer launches (qtts.h qtts_session_set_wait_budget)."""
        _check(lib.qtts_session_set_wait_budget(self.h, int(ns)))

    def close(self):
        if getattr(self, "h", None):
            lib.qtts_session_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def frame_kernel_count(self) -> int:
        return lib.qtts_frame_kernel_count(self.h)

    def graph_captures(self) -> int:
        """Frame graphs captured so far (a generation of an unchanged shape
        reuses the last one)."""
        return lib.qtts_frame_graph_captures(self.h)

    def family_time(self, family: int, reps: int = 50) -> dict:
        """Profiling: device time of one frame's launches of one kernel
        family replayed alone (qtts.h qtts_frame_family_time).  Ends the
        generation in progress."""
        ms, n = C.c_float(), C.c_int()
        fl, wb = C.c_double(), C.c_double()
        _check(lib.qtts_frame_family_time(self.h, family, reps, C.byref(ms), C.byref(n), C.byref(fl), C.byref(wb)))
        return {"ms": ms.value, "launches": n.value, "flops": fl.value, "weight_bytes": wb.value}


# ---- reference-facing functions (talker.rs / code_predictor.rs / generate_new.rs)

def embed_text_token(sess: Session, token_id: int) -> np.ndarray:
    """talker.rs:105 embed_text_token."""
    out = np.zeros(sess.H, np.float32)
    _check(lib.qtts_embed_text(sess.h, token_id, _fp(out)))
    return out


def embed_codec_token(sess: Session, token_id: int) -> np.ndarray:
    """talker.rs:152 embed_codec_token."""
    out = np.zeros(sess.H, np.float32)
    _check(lib.qtts_embed_codec(sess.h, token_id, _fp(out)))
    return out


def prefill_talker_raw(sess: Session, x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """talker.rs:364 prefill_talker_raw (+ talker.rs:627 apply_codec_head on
    the returned hidden).  Returns (last_hidden, logits)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, sess.H)
    hid = np.zeros(sess.H, np.float32)
    lg = np.zeros(sess.V, np.float32)
    _check(lib.qtts_prefill(sess.h, _fp(x), x.shape[0], _fp(hid), _fp(lg)))
    return hid, lg


def forward_with_embedding(sess: Session, embedding: np.ndarray, position: int) -> np.ndarray:
    """talker.rs:263 forward_with_embedding -> [normed_hidden ++ logits]."""
    emb = np.ascontiguousarray(embedding, np.float32)
    out = np.zeros(sess.H + sess.V, np.float32)
    _check(lib.qtts_talker_step(sess.h, _fp(emb), position, _fp(out)))
    return out


def generate_acoustic_codes(sess: Session, talker_hidden: np.ndarray, semantic_embed: np.ndarray) -> np.ndarray:
    """code_predictor.rs:218 generate_acoustic_codes (resets the predictor cache)."""
    codes = np.zeros(sess.dims.p_groups, np.uint32)
    _check(lib.qtts_predict_acoustic(sess.h, _fp(np.ascontiguousarray(talker_hidden, np.float32)),
                                     _fp(np.ascontiguousarray(semantic_embed, np.float32)), _u32p(codes)))
    return codes


def get_acoustic_embeddings_sum(sess: Session, acoustic_codes) -> np.ndarray:
    """code_predictor.rs:280 get_acoustic_embeddings_sum."""
    codes = np.ascontiguousarray(acoustic_codes, np.uint32)
    out = np.zeros(sess.H, np.float32)
    _check(lib.qtts_acoustic_embed_sum(sess.h, _u32p(codes), _fp(out)))
    return out


def sample_token(sess: Session, logits, params: SampleParams, prev_tokens, rng_state: int) -> tuple[int, int]:
    """generate_new.rs:329 sample_token -> (token, advanced rng state)."""
    lg = np.ascontiguousarray(logits, np.float32)
    prev = np.ascontiguousarray(prev_tokens, np.uint32)
    st = C.c_uint64(rng_state)
    out = np.zeros(1, np.uint32)
    _check(lib.qtts_sample(sess.h, _fp(lg), lg.size, C.byref(params), _u32p(prev), C.byref(st), _u32p(out)))
    return int(out[0]), st.value


def make_params(temperature=1.0, top_k=1, repetition_penalty=1.05, codec_eos_id=2150) -> SampleParams:
    return SampleParams(temperature, top_k, repetition_penalty, codec_eos_id)


class _Utts:
    """Keeps the numpy buffers behind a ctypes Utterance array alive."""

    def __init__(self, utterances):
        self.keep = []
        arr = (Utterance * len(utterances))()
        for i, u in enumerate(utterances):
            text = np.ascontiguousarray(u["text"], np.uint32)
            self.keep.append(text)
            arr[i].text = _u32p(text)
            arr[i].n_text = int(text.size)
            arr[i].speaker_id = int(u.get("speaker_id", 0))
            arr[i].language_id = int(u.get("language_id", 2050))
            v = u.get("voice")
            if v is not None:
                v = np.ascontiguousarray(v, np.float32)
                self.keep.append(v)
                arr[i].voice = _fp(v)
            arr[i].seed = int(u.get("seed", 0))
            p = u.get("params") or make_params()
            arr[i].params = p
        self.arr = arr
        self.n = len(utterances)


def _flags(ignore_eos: bool, full_prompt: bool) -> int:
    return (IGNORE_EOS if ignore_eos else 0) | (FULL_PROMPT if full_prompt else 0)


def generate(sess: Session, utterances, max_frames: int, ignore_eos: bool = True, forced=None,
             dump_logits: bool = False, dump_hidden: bool = False, full_prompt: bool = False):
    """The generate_new.rs:191-300 frame loop for a batch of utterances.

    Each utterance is a dict(text=token ids, voice=None|[H], speaker_id,
    language_id, seed, params=SampleParams).  full_prompt: the benchmark mode
    that prefills the whole text (ragged KV lengths; qtts.h QTTS_FULL_PROMPT).
    Returns (codes [n][F][16], frames [n], logits [n][F][V] | None,
    hidden [n][F][H] | None)."""
    u = _Utts(utterances)
    n = u.n
    codes = np.zeros((n, max_frames, 16), np.uint32)
    frames = np.zeros(n, np.int32)
    lg = np.zeros((n, max_frames, sess.V), np.float32) if dump_logits else None
    hd = np.zeros((n, max_frames, sess.H), np.float32) if dump_hidden else None
    fc = None if forced is None else np.ascontiguousarray(forced, np.uint32).reshape(n, max_frames, 16)
    _check(lib.qtts_generate(sess.h, n, u.arr, max_frames, _flags(ignore_eos, full_prompt),
                             _u32p(fc) if fc is not None else None, _u32p(codes),
                             frames.ctypes.data_as(C.POINTER(C.c_int)),
                             _fp(lg) if lg is not None else None, _fp(hd) if hd is not None else None))
    return codes, frames, lg, hd


class Generation:
    """generate() split for timing: begin (prefill + graph capture), frames
    (asynchronous graph replays on the session stream), end (sync + copy)."""

    def __init__(self, sess: Session, utterances, max_frames: int, ignore_eos: bool = True, forced=None,
                 full_prompt: bool = False):
        self.sess = sess
        self.u = _Utts(utterances)
        self.max_frames = max_frames
        self.forced = None if forced is None else np.ascontiguousarray(forced, np.uint32)
        _check(lib.qtts_generate_begin(sess.h, self.u.n, self.u.arr, max_frames,
                                       _flags(ignore_eos, full_prompt),
                                       _u32p(self.forced) if self.forced is not None else None))

    def frames(self, n: int):
        _check(lib.qtts_generate_frames(self.sess.h, n))

    def end(self):
        codes = np.zeros((self.u.n, self.max_frames, 16), np.uint32)
        frames = np.zeros(self.u.n, np.int32)
        _check(lib.qtts_generate_end(self.sess.h, _u32p(codes), frames.ctypes.data_as(C.POINTER(C.c_int)),
                                     None, None))
        return codes, frames


# ---- kernel-level entry points (gemv.rs:149 gemv, :157 gemm) ------------------

def q4_gemv(packed: np.ndarray, scales: np.ndarray, k: int, n: int, x: np.ndarray) -> np.ndarray:
    """Host-buffer Q4 GEMV/GEMM: y[m][n] = x[m][k] @ W (W in the on-disk layout)."""
    x = np.ascontiguousarray(x, np.float32).reshape(-1, k)
    y = np.zeros((x.shape[0], n), np.float32)
    _check(lib.qtts_q4_gemv(packed.ctypes.data_as(C.POINTER(C.c_uint8)),
                            scales.ctypes.data_as(C.POINTER(C.c_uint16)), k, n, _fp(x), x.shape[0], _fp(y)))
    return y


def q4_gemv_scratch_bytes(k: int, n: int, m: int) -> int:
    return int(lib.qtts_q4_gemv_scratch_bytes(k, n, m))


def q4_gemv_dev(packed_ptr, scales_ptr, k, n, x_ptr, m, y_ptr, scratch_ptr, scratch_bytes, stream=0):
    _check(lib.qtts_q4_gemv_dev(packed_ptr, scales_ptr, k, n, x_ptr, m, y_ptr, scratch_ptr, scratch_bytes,
                                stream or None))


def f16_gemv_dev(w_ptr, k, n, x_ptr, m, y_ptr, stream=0):
    _check(lib.qtts_f16_gemv_dev(w_ptr, k, n, x_ptr, m, y_ptr, stream or None))


def q4_dequant_dev(packed_ptr, scales_ptr, k, n, out_ptr, stream=0):
    _check(lib.qtts_q4_dequant_dev(packed_ptr, scales_ptr, k, n, out_ptr, stream or None))


def quantize_f32_to_q4(data: np.ndarray, k: int, n: int) -> tuple[np.ndarray, np.ndarray]:
    """gemv.rs:92-130 on the GPU: f32 [k][n] -> (packed u8 [k*n/2], scales f16 bits u16 [k*n/32])."""
    d = np.ascontiguousarray(data, np.float32).reshape(-1)
    if d.size != k * n:
        raise QttsError(ERR_BADARG, f"data has {d.size} values, expected {k}*{n}")
    packed = np.empty(k * n // 2, np.uint8)
    scales = np.empty(k * n // 32, np.uint16)
    _check(lib.qtts_q4_quantize(_fp(d), k, n, packed.ctypes.data_as(C.POINTER(C.c_uint8)),
                                scales.ctypes.data_as(C.POINTER(C.c_uint16))))
    return packed, scales


def q4_quantize_dev(data_ptr, k, n, packed_ptr, scales_ptr, stream=0):
    _check(lib.qtts_q4_quantize_dev(data_ptr, k, n, packed_ptr, scales_ptr, stream or None))


def expf_dev(x_ptr, y_ptr, n, stream=0):
    """The sampler's exp (bit-identical to glibc expf), for validation."""
    _check(lib.qtts_expf_dev(x_ptr, y_ptr, n, stream or None))
