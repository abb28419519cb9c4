"""CPU tests of the speech decoder's first stage (decoder.rs:142-335 with the
conv.rs:114-191 pre-conv): the synthetic decoder section written by the
library and by the oracle is the same file; the library's reader accepts it;
and the C oracle's restatement agrees with a second, numpy restatement of
the same steps on a few frames (an independent check of its structure:
codebook sums, the causal taps, RoPE positions, the 72-frame window, the
layer scales).  No GPU needed."""
import hashlib

import numpy as np
import pytest

H, A, I, CB, HD, HEADS, WIN = 512, 1024, 1024, 256, 64, 16, 72


def _sha(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for b in iter(lambda: f.read(1 << 22), b""):
            h.update(b)
    return h.hexdigest()


@pytest.fixture(scope="module")
def dec_file(qtts, tmp_path_factory):
    p = str(tmp_path_factory.mktemp("dec") / "prod.qora-tts")
    qtts.synth_write_with_decoder(p, qtts.dims_tiny(), 11)
    return p


def test_decoder_writer_matches_oracle_writer(qtts, oracle_mod, dec_file, tmp_path):
    b = str(tmp_path / "orc.qora-tts")
    oracle_mod.synth_write_with_decoder(b, oracle_mod.dims_tiny(), 11)
    assert _sha(dec_file) == _sha(b)


def test_decoder_file_keeps_talker_and_predictor(qtts, dec_file, tmp_path):
    # the decoder section follows the predictor: the bytes before it, and the
    # dims the reader derives, are those of the file without a decoder
    plain = str(tmp_path / "plain.qora-tts")
    qtts.synth_write(plain, qtts.dims_tiny(), 11)
    # the empty decoder section: 17 u32 counts / headers (68 B), 23 empty vectors (184 B),
    # the conv headers of pre-conv, vocos_init and output_conv inside those
    n = len(open(plain, "rb").read()) - 256
    with open(plain, "rb") as f, open(dec_file, "rb") as g:
        assert f.read(n) == g.read(n)
        assert g.read(24) == np.array([H, HEADS, HD, I, WIN, CB], "<u4").tobytes()
    assert qtts.file_probe(dec_file).as_dict() == qtts.dims_tiny().as_dict()


def test_synth_flags_rejected(qtts, tmp_path):
    import ctypes as C
    rc = qtts.lib.qtts_synth_write_ex(str(tmp_path / "x").encode(), C.byref(qtts.dims_tiny()), 1, 0x10)
    assert rc == qtts.ERR_BADARG


def _read_decoder(path):
    """save.rs:446-552 on the numpy side: the decoder section's tensors."""
    import struct
    with open(path, "rb") as f:
        data = f.read()
    # find the decoder header (six u32: 512, 16, 64, 1024, 72, 256) after the predictor
    hdr = struct.pack("<6I", H, HEADS, HD, I, WIN, CB)
    pos = data.rindex(hdr)
    at = pos + 24

    def vec():
        nonlocal at
        n = struct.unpack_from("<Q", data, at)[0]
        at += 8
        v = np.frombuffer(data, np.float32, n, at).copy()
        at += 4 * n
        return v

    def u32():
        nonlocal at
        v = struct.unpack_from("<I", data, at)[0]
        at += 4
        return v

    d = {"cb0": vec().reshape(-1, CB), "p0": vec().reshape(CB, 512)}
    assert u32() == 15
    d["cbr"] = [vec().reshape(-1, CB) for _ in range(15)]
    d["pr"] = vec().reshape(CB, 512)
    hdr6 = [u32() for _ in range(6)]
    d["pre_w"] = vec().reshape(hdr6[1], hdr6[0], hdr6[2])
    d["pre_b"] = vec()
    d["in_w"] = vec().reshape(1024, H)
    d["in_b"] = vec()
    d["layers"] = []
    for _ in range(u32()):
        names = ["q", "k", "v", "o", "gate", "up", "down", "n1", "n2", "s1", "s2"]
        d["layers"].append({k: vec() for k in names})
    d["norm"], d["out_w"], d["out_b"] = vec(), vec().reshape(H, 1024), vec()
    assert u32() == 0  # no upsample stages
    [u32() for _ in range(6)], vec(), vec()
    assert u32() == 0  # no vocos blocks
    vec(), vec(), [u32() for _ in range(6)], vec(), vec()
    d["cos"], d["sin"] = vec().reshape(-1, HD // 2), vec().reshape(-1, HD // 2)
    return d


def _numpy_decode(d, codes):
    f32 = np.float32
    T = codes.shape[1]
    vq = d["cb0"][codes[0]] @ d["p0"]
    vq = vq + (sum(d["cbr"][g][codes[g + 1]] for g in range(15)) @ d["pr"])
    xp = np.concatenate([np.zeros((2, 512), f32), vq])  # causal left pad (k - 1) = 2
    pre = d["pre_b"] + sum(xp[k:k + T] @ d["pre_w"][:, :, k].T for k in range(3))
    x = pre @ d["in_w"] + d["in_b"]

    def rms(v, g):
        return v / np.sqrt((v * v).sum(-1, keepdims=True) / v.shape[-1] + 1e-5) * g

    def rope(m):
        m = m.reshape(T, HEADS, HD).copy()
        c, s = d["cos"][:T, None, :], d["sin"][:T, None, :]
        x0, x1 = m[..., :HD // 2].copy(), m[..., HD // 2:].copy()
        m[..., :HD // 2] = x0 * c - x1 * s
        m[..., HD // 2:] = x1 * c + x0 * s
        return m

    for L in d["layers"]:
        xn = rms(x, L["n1"])
        q, k = rope(xn @ L["q"].reshape(H, A)), rope(xn @ L["k"].reshape(H, A))
        v = (xn @ L["v"].reshape(H, A)).reshape(T, HEADS, HD)
        ao = np.zeros((T, HEADS, HD), f32)
        for t in range(T):
            s0 = max(0, t + 1 - WIN)
            sc = np.einsum("hd,shd->hs", q[t], k[s0:t + 1]) / np.sqrt(f32(HD))
            p = np.exp(sc - sc.max(-1, keepdims=True))
            p /= p.sum(-1, keepdims=True)
            ao[t] = np.einsum("hs,shd->hd", p, v[s0:t + 1])
        x = x + (ao.reshape(T, A) @ L["o"].reshape(A, H)) * L["s1"]
        xn = rms(x, L["n2"])
        g, u = xn @ L["gate"].reshape(H, I), xn @ L["up"].reshape(H, I)
        x = x + (((g / (1 + np.exp(-g))) * u) @ L["down"].reshape(I, H)) * L["s2"]
    return (rms(x, d["norm"]) @ d["out_w"] + d["out_b"]).T


@pytest.mark.parametrize("T", [3, 80])
def test_oracle_decoder_matches_numpy_restatement(oracle_mod, dec_file, T):
    # T = 80 crosses the 72-frame attention window
    codes = np.random.default_rng(T).integers(0, 2048, (16, T)).astype(np.uint32)
    dec = oracle_mod.Decoder(dec_file)
    got = dec.decode_latent(codes)
    dec.close()
    ref = _numpy_decode(_read_decoder(dec_file), codes.astype(np.int64))
    err = float(np.max(np.abs(got - ref)) / np.max(np.abs(ref)))
    assert err < 1e-4, err


def test_oracle_decoder_rejects_bad_code(oracle_mod, dec_file):
    dec = oracle_mod.Decoder(dec_file)
    codes = np.zeros((16, 4), np.uint32)
    codes[7, 2] = 2048
    with pytest.raises(ValueError):
        dec.decode_latent(codes)
    dec.close()


def test_oracle_decoder_load_needs_a_decoder(oracle_mod, tiny_path):
    with pytest.raises(IOError):
        oracle_mod.Decoder(tiny_path)


def test_truncated_decoder_section_rejected(qtts, oracle_mod, dec_file, tmp_path):
    # cut inside the decoder's transformer weights: the reader walks the
    # whole section (save.rs:446-552), so the file is refused as the
    # reference's loader would refuse it, by the library and by the oracle
    data = open(dec_file, "rb").read()
    bad = str(tmp_path / "cut.qora-tts")
    with open(bad, "wb") as f:
        f.write(data[: len(data) - 60_000_000])
    with pytest.raises(qtts.QttsError) as e:
        qtts.file_probe(bad)
    assert e.value.code == qtts.ERR_FORMAT
    with pytest.raises(IOError):
        oracle_mod.Decoder(bad)
