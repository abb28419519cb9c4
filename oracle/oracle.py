"""ctypes binding of the CPU oracle (oracle/qtts_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by bench.py's ``cpu_baseline`` / ``--impl reference`` legs, always as the
checker or the timed CPU baseline, never as the product path.

Parity status: UNPINNED.  The reference is a Rust crate that cannot be built
in this image, and its tests hold no golden vectors for the decode loop; the
restatement follows the reference file:line citations in qtts_oracle.c.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")


def build(force: bool = False) -> str:
    """Compile liboracle.so with the committed Makefile (gcc only)."""
    src = os.path.join(HERE, "qtts_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE])
    return LIB_PATH


class Dims(C.Structure):
    _fields_ = [(n, C.c_int) for n in (
        "t_layers", "t_hidden", "t_text_hidden", "t_heads", "t_kv_heads", "t_head_dim",
        "t_inter", "t_vocab", "t_text_vocab", "t_max_pos")] + [("t_sec", C.c_int * 3)] + [
        (n, C.c_int) for n in ("p_layers", "p_hidden", "p_heads", "p_kv_heads", "p_head_dim",
                               "p_inter", "p_vocab", "p_groups", "p_max_pos", "fmt")]


class Params(C.Structure):
    _fields_ = [("max_codes", C.c_int), ("temperature", C.c_float), ("top_k", C.c_int),
                ("repetition_penalty", C.c_float), ("codec_eos_id", C.c_uint32),
                ("codec_bos_id", C.c_uint32)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        build()
        L = C.CDLL(LIB_PATH)
        P = C.c_void_p
        fp = C.POINTER(C.c_float)
        u8p = C.POINTER(C.c_uint8)
        u16p = C.POINTER(C.c_uint16)
        u32p = C.POINTER(C.c_uint32)
        u64p = C.POINTER(C.c_uint64)
        sz = C.c_size_t
        sig = {
            "oq_h2f": (C.c_float, [C.c_uint16]),
            "oq_f2h": (C.c_uint16, [C.c_float]),
            "oq_synth_write": (C.c_int, [C.c_char_p, C.POINTER(Dims), C.c_uint64]),
            "oq_set_tie_period": (None, [C.c_int]),
            "oq_dims_1p7b": (None, [C.POINTER(Dims)]),
            "oq_dims_tiny": (None, [C.POINTER(Dims)]),
            "oq_load": (P, [C.c_char_p, C.c_char_p, C.c_int]),
            "oq_free": (None, [P]),
            "oq_get_dims": (None, [P, C.POINTER(Dims)]),
            "oq_set_threads": (None, [C.c_int]),
            "oq_get_threads": (C.c_int, []),
            "oq_gemv_q4": (None, [fp, u8p, u16p, sz, sz, fp]),
            "oq_gemm_q4": (None, [fp, sz, u8p, u16p, sz, sz, fp]),
            "oq_gemv_f16": (None, [fp, u16p, sz, sz, fp]),
            "oq_quantize_q4": (None, [fp, sz, sz, u8p, u16p]),
            "oq_embed_q4": (None, [u8p, u16p, sz, sz, fp]),
            "oq_rms_norm_f16": (None, [fp, u16p, sz, fp]),
            "oq_softmax_raw": (None, [fp, sz]),
            "oq_silu": (C.c_float, [C.c_float]),
            "oq_build_mrope_tables": (None, [C.c_int, C.c_int, C.c_double, C.POINTER(C.c_int), C.c_int, fp, fp]),
            "oq_build_rope_tables": (None, [C.c_int, C.c_int, C.c_double, fp, fp]),
            "oq_kv_free": (None, [P]),
            "oq_kv_clear": (None, [P]),
            "oq_kv_len": (C.c_int, [P, C.c_int]),
            "oq_talker_kv_new": (P, [P]),
            "oq_predictor_kv_new": (P, [P]),
            "oq_embed_text_token": (None, [P, C.c_uint32, fp]),
            "oq_embed_codec_token": (None, [P, C.c_uint32, fp]),
            "oq_forward_with_embedding": (C.c_int, [P, fp, P, C.c_int, fp]),
            "oq_prefill_talker_raw": (C.c_int, [P, fp, C.c_int, P, fp]),
            "oq_apply_codec_head": (None, [P, fp, fp]),
            "oq_generate_acoustic_codes": (None, [P, fp, fp, P, u32p]),
            "oq_acoustic_embed_sum": (None, [P, u32p, fp]),
            "oq_sample_argmax": (C.c_uint32, [fp, sz]),
            "oq_simple_rand": (C.c_float, [u64p]),
            "oq_sample_token": (C.c_uint32, [fp, sz, C.POINTER(Params), u32p, u64p]),
            "oq_prefill_custom_voice": (C.c_int, [P, u32p, C.c_int, C.c_uint32, C.c_uint32, fp, P, fp, fp]),
            "oq_generate": (C.c_int, [P, u32p, C.c_int, C.c_uint32, C.c_uint32, fp, C.POINTER(Params),
                                      C.c_uint64, C.c_int, u32p, u32p, fp, fp]),
            "oq_time_frames": (C.c_double, [P, C.c_int, C.c_int, C.c_uint64]),
            "oq_synth_write_ex": (C.c_int, [C.c_char_p, C.POINTER(Dims), C.c_uint64, C.c_uint]),
            "oq_decoder_load": (P, [C.c_char_p, C.c_char_p, C.c_int]),
            "oq_decoder_free": (None, [P]),
            "oq_decode_latent": (C.c_int, [P, u32p, C.c_int, fp]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def _p(a, ct):
    return a.ctypes.data_as(C.POINTER(ct)) if a is not None else None


def fptr(a):
    return _p(a, C.c_float)


def dims_1p7b() -> Dims:
    d = Dims()
    lib().oq_dims_1p7b(C.byref(d))
    return d


def dims_tiny() -> Dims:
    d = Dims()
    lib().oq_dims_tiny(C.byref(d))
    return d


def synth_write(path: str, dims: Dims, seed: int = 0) -> None:
    rc = lib().oq_synth_write(path.encode(), C.byref(dims), seed)
    if rc != 0:
        raise IOError(f"oracle synth_write failed for {path}")


SYNTH_DECODER = 1


def synth_write_with_decoder(path: str, dims: Dims, seed: int = 0) -> None:
    """The synthetic model with a full-size speech decoder section
    (codebooks, pre-conv, transformer, RoPE; upsample / Vocos empty)."""
    rc = lib().oq_synth_write_ex(path.encode(), C.byref(dims), seed, SYNTH_DECODER)
    if rc != 0:
        raise IOError(f"oracle synth_write_ex failed for {path}")


class Decoder:
    """decoder.rs:142-335 + the conv.rs:114-191 pre-conv on the CPU: 16 code
    streams of T frames -> the transformer output [1024][T]."""

    def __init__(self, path: str):
        err = C.create_string_buffer(256)
        self.h = lib().oq_decoder_load(path.encode(), err, 256)
        if not self.h:
            raise IOError(f"oracle decoder load failed: {err.value.decode()}")

    def decode_latent(self, codes):
        import numpy as np
        codes = np.ascontiguousarray(codes, dtype=np.uint32)
        assert codes.ndim == 2 and codes.shape[0] == 16
        T = codes.shape[1]
        out = np.zeros((1024, T), np.float32)
        rc = lib().oq_decode_latent(self.h, _p(codes, C.c_uint32), T, fptr(out))
        if rc != 0:
            raise ValueError("code index past its codebook")
        return out

    def close(self):
        if getattr(self, "h", None):
            lib().oq_decoder_free(self.h)
            self.h = None

    def __del__(self):
        self.close()


def synth_write_tied_heads(path: str, dims: Dims, seed: int = 0, period: int = 7) -> None:
    """Test fixture: the synthetic model with every predictor head's column j
    equal to column j % period (bit-equal logits in each residue class, so
    the greedy argmax meets exact ties)."""
    lib().oq_set_tie_period(period)
    try:
        synth_write(path, dims, seed)
    finally:
        lib().oq_set_tie_period(0)


def set_threads(n: int) -> None:
    lib().oq_set_threads(int(n))


# --- raw kernels ------------------------------------------------------------

def gemv_q4(x, packed, scales, k, n):
    y = np.zeros(n, np.float32)
    lib().oq_gemv_q4(fptr(x), _p(packed, C.c_uint8), _p(scales, C.c_uint16), k, n, fptr(y))
    return y


def gemm_q4(x, packed, scales, k, n):
    seq = x.shape[0]
    y = np.zeros((seq, n), np.float32)
    lib().oq_gemm_q4(fptr(np.ascontiguousarray(x, np.float32)), seq, _p(packed, C.c_uint8),
                     _p(scales, C.c_uint16), k, n, fptr(y))
    return y


def gemv_f16(x, w, k, n):
    y = np.zeros(n, np.float32)
    lib().oq_gemv_f16(fptr(x), _p(w, C.c_uint16), k, n, fptr(y))
    return y


def quantize_q4(data, k, n):
    packed = np.zeros(k * n // 2, np.uint8)
    scales = np.zeros(k * n // 32, np.uint16)
    lib().oq_quantize_q4(fptr(np.ascontiguousarray(data, np.float32)), k, n, _p(packed, C.c_uint8),
                         _p(scales, C.c_uint16))
    return packed, scales


def embed_q4(packed, scales, n, row):
    out = np.zeros(n, np.float32)
    lib().oq_embed_q4(_p(packed, C.c_uint8), _p(scales, C.c_uint16), n, row, fptr(out))
    return out


def sample_argmax(logits):
    logits = np.ascontiguousarray(logits, np.float32)
    return int(lib().oq_sample_argmax(fptr(logits), logits.size))


def simple_rand(state: int):
    st = C.c_uint64(state)
    r = lib().oq_simple_rand(C.byref(st))
    return r, st.value


def make_params(max_codes=100, temperature=1.0, top_k=1, repetition_penalty=1.05,
                codec_eos_id=2150, codec_bos_id=2149) -> Params:
    return Params(max_codes, temperature, top_k, repetition_penalty, codec_eos_id, codec_bos_id)


def sample_token(logits, params: Params, prev16, rng_state: int):
    logits = np.ascontiguousarray(logits, np.float32)
    prev = np.ascontiguousarray(prev16, np.uint32)
    st = C.c_uint64(rng_state)
    tok = lib().oq_sample_token(fptr(logits), logits.size, C.byref(params), _p(prev, C.c_uint32),
                                C.byref(st))
    return int(tok), st.value


class Model:
    """A loaded .qora-tts file on the CPU (talker + code predictor)."""

    def __init__(self, path: str):
        err = C.create_string_buffer(256)
        self.h = lib().oq_load(path.encode(), err, 256)
        if not self.h:
            raise IOError(err.value.decode())
        self.dims = Dims()
        lib().oq_get_dims(self.h, C.byref(self.dims))
        self.H = self.dims.t_hidden
        self.V = self.dims.t_vocab

    def close(self):
        if self.h:
            lib().oq_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def talker_kv(self):
        return KV(lib().oq_talker_kv_new(self.h))

    def predictor_kv(self):
        return KV(lib().oq_predictor_kv_new(self.h))

    def embed_text_token(self, tok):
        out = np.zeros(self.dims.t_hidden, np.float32)
        lib().oq_embed_text_token(self.h, tok, fptr(out))
        return out

    def embed_codec_token(self, tok):
        out = np.zeros(self.dims.t_hidden, np.float32)
        lib().oq_embed_codec_token(self.h, tok, fptr(out))
        return out

    def forward_with_embedding(self, emb, kv, position):
        out = np.zeros(self.H + self.V, np.float32)
        emb = np.ascontiguousarray(emb, np.float32)
        rc = lib().oq_forward_with_embedding(self.h, fptr(emb), kv.h, position, fptr(out))
        if rc:
            raise IndexError("position beyond the rope table")
        return out

    def prefill_talker_raw(self, x, kv):
        x = np.ascontiguousarray(x, np.float32)
        out = np.zeros(self.H, np.float32)
        rc = lib().oq_prefill_talker_raw(self.h, fptr(x), x.shape[0], kv.h, fptr(out))
        if rc:
            raise IndexError("position beyond the rope table")
        return out

    def apply_codec_head(self, h):
        out = np.zeros(self.V, np.float32)
        lib().oq_apply_codec_head(self.h, fptr(np.ascontiguousarray(h, np.float32)), fptr(out))
        return out

    def generate_acoustic_codes(self, talker_hidden, semantic_embed, pkv):
        codes = np.zeros(self.dims.p_groups, np.uint32)
        lib().oq_generate_acoustic_codes(self.h, fptr(np.ascontiguousarray(talker_hidden, np.float32)),
                                         fptr(np.ascontiguousarray(semantic_embed, np.float32)), pkv.h,
                                         _p(codes, C.c_uint32))
        return codes

    def acoustic_embed_sum(self, codes):
        codes = np.ascontiguousarray(codes, np.uint32)
        out = np.zeros(self.dims.t_hidden, np.float32)
        lib().oq_acoustic_embed_sum(self.h, _p(codes, C.c_uint32), fptr(out))
        return out

    def prefill_custom_voice(self, text, speaker_id, language_id, voice, kv):
        text = np.ascontiguousarray(text, np.uint32)
        hid = np.zeros(self.H, np.float32)
        lg = np.zeros(self.V, np.float32)
        v = None if voice is None else np.ascontiguousarray(voice, np.float32)
        seq = lib().oq_prefill_custom_voice(self.h, _p(text, C.c_uint32), text.size, speaker_id,
                                            language_id, fptr(v) if v is not None else None, kv.h,
                                            fptr(hid), fptr(lg))
        return seq, hid, lg

    def generate(self, text, params: Params, seed: int, speaker_id=0, language_id=2050, voice=None,
                 ignore_eos=True, forced=None, dump_logits=False, dump_hidden=False, full_prompt=False):
        text = np.ascontiguousarray(text, np.uint32)
        F = params.max_codes
        codes = np.zeros((F, 16), np.uint32)
        lg = np.zeros((F, self.V), np.float32) if dump_logits else None
        hd = np.zeros((F, self.H), np.float32) if dump_hidden else None
        fc = None if forced is None else np.ascontiguousarray(forced, np.uint32)
        v = None if voice is None else np.ascontiguousarray(voice, np.float32)
        n = lib().oq_generate(self.h, _p(text, C.c_uint32), text.size, speaker_id, language_id,
                              fptr(v) if v is not None else None, C.byref(params), seed,
                              (1 if ignore_eos else 0) | (2 if full_prompt else 0),
                              _p(fc, C.c_uint32) if fc is not None else None,
                              _p(codes, C.c_uint32), fptr(lg) if lg is not None else None,
                              fptr(hd) if hd is not None else None)
        if n < 0:
            raise RuntimeError("oracle generate failed")
        return n, codes, lg, hd

    def time_frames(self, kv_len, frames, seed=7):
        return lib().oq_time_frames(self.h, kv_len, frames, seed)


class KV:
    def __init__(self, h):
        self.h = h

    def clear(self):
        lib().oq_kv_clear(self.h)

    def len(self, layer=0):
        return lib().oq_kv_len(self.h, layer)

    def __del__(self):
        try:
            if self.h:
                lib().oq_kv_free(self.h)
                self.h = None
        except Exception:
            pass
