"""NPRTCKPTV2 / V3 checkpoint codec on CPU.

Three implementations are compared byte for byte: the product codec in
libhexatrain_b200.so (hexatrain_b200.checkpoint), the oracle's C restatement
of the writer, and the reference's own nprtSaveCheckpointV2 /
nprtLoadCheckpointForGeneration (qnn/qnn_transformer_training.cpp:5171-5252,
:5390-5522) compiled from its sources into oracle/_ref/libhexaref_ckpt.so.
Every reader rejection is checked against the reference reader's own error
code on the same bytes; the cases follow the reference's resume test
(host_tests/nicopedia_resume_test.cpp: round trip, V1 without Adam, step and
seed mismatches, configuration mismatches) and its reader's checks.
"""
import os
import struct

import numpy as np
import pytest

import hexatrain_b200 as hx
from hexatrain_b200 import checkpoint as ck
from oracle.oracle import LmConfig as OC
from oracle.oracle import ReferenceCheckpoint, reference_checkpoint_available

HASH = "sha256:" + "0123456789abcdef" * 4
CONFIGS = [
    # (V, T, D, F, L, H), tokenizer identity or None
    ((32, 4, 8, 16, 2, 2), None),
    ((40, 6, 8, 12, 3, 2), None),
    ((1024, 8, 16, 16, 1, 2), ("byte_bpe", HASH)),
]

needs_ref = pytest.mark.skipif(not reference_checkpoint_available(),
                               reason="reference checkpoint codec (oracle/_ref/libhexaref_ckpt.so) not built")


@pytest.fixture(scope="module")
def ref():
    if not reference_checkpoint_available():
        pytest.skip("reference checkpoint codec not built")
    return ReferenceCheckpoint()


def _state(n, seed):
    rng = np.random.default_rng(seed)
    p = rng.standard_normal(n).astype(np.float32)
    m = (rng.standard_normal(n) * 1e-3).astype(np.float32)
    v = (rng.random(n) * 1e-6).astype(np.float32)
    return p, m, v


def _cfgs(dims, learned=False):
    V, T, D, F, L, H = dims
    return hx.LmConfig(V, T, D, F, L, H, learned_position=learned), OC.make(V, T, D, F, L, H,
                                                                             learned_position=learned)


@needs_ref
@pytest.mark.parametrize("dims,tok", CONFIGS, ids=["V32_L2", "V40_L3", "V1024_L1_v3"])
def test_three_writers_agree_byte_for_byte(dims, tok, ref, oracle, tmp_path):
    cfg, oc = _cfgs(dims)
    n = cfg.parameter_count()
    p, m, v = _state(n, 11)
    kind, hsh = tok if tok else (None, None)
    path = str(tmp_path / "ref.ckpt")
    assert ref.save(path, oc, 20260710, 12, p, m, v, kind, hsh)
    want = open(path, "rb").read()
    assert want[:11] == (b"NPRTCKPTV3\n" if tok else b"NPRTCKPTV2\n")
    assert oracle.nprt_encode(oc, 20260710, 12, p, m, v, kind, hsh) == want
    assert ck.encode(cfg, 20260710, 12, p, m, v, kind, hsh) == want


@needs_ref
@pytest.mark.parametrize("dims,tok", CONFIGS, ids=["V32_L2", "V40_L3", "V1024_L1_v3"])
def test_decode_round_trips_against_the_reference_reader(dims, tok, ref, tmp_path):
    cfg, oc = _cfgs(dims)
    n = cfg.parameter_count()
    p, m, v = _state(n, 12)
    kind, hsh = tok if tok else (None, None)
    data = ck.encode(cfg, 7, 25, p, m, v, kind, hsh)
    info, p2, m2, v2 = ck.decode(cfg, data, 7, hsh)
    assert info.step == 25 and info.has_adam and info.finite and info.version == (3 if tok else 2)
    assert np.array_equal(p2, p) and np.array_equal(m2, m) and np.array_equal(v2, v)
    path = str(tmp_path / "ours.ckpt")
    open(path, "wb").write(data)
    ok, err, rinfo, rp, rm, rv = ref.load(path, oc, 7, n, hsh)
    assert ok, err
    assert rinfo["step"] == 25 and rinfo["has_adam"] and rinfo["finite"]
    assert np.array_equal(rp, p) and np.array_equal(rm, m) and np.array_equal(rv, v)
    assert rinfo["parameter_hash"] == info.parameter_hash == ref.parameter_hash(oc, p)


def _mutations(data, dims, tok):
    """(label, bytes) variants of a valid file, each one a reader check."""
    V = dims[0]
    head = 11 + 8 * 4 + ((4 + 8 + 4 + 71) if tok else 0)
    reg0 = head + 4                      # first registry entry
    name_len = struct.unpack(">I", data[reg0:reg0 + 4])[0]
    out = [
        ("bad magic", b"NPRTCKPTV9\n" + data[11:]),
        ("step 0", data[:11 + 28] + struct.pack(">I", 0) + data[11 + 32:]),
        ("step 1e6", data[:11 + 28] + struct.pack(">I", 1000000) + data[11 + 32:]),
        ("trailing byte", data + b"\0"),
        ("truncated values", data[:-5]),
        ("truncated header", data[:20]),
        ("name length 0", data[:reg0] + struct.pack(">I", 0) + data[reg0 + 4:]),
        ("registry order", data[:reg0 + 4] + b"x" + data[reg0 + 5:]),
        ("element count", data[:reg0 + 4 + name_len] + struct.pack(">Q", 3) + data[reg0 + 12 + name_len:]),
        ("registry count", data[:head] + struct.pack(">I", 5) + data[head + 4:]),
    ]
    if tok:
        out.append(("v2 magic at vocabulary 1024",
                    b"NPRTCKPTV2\n" + data[11:11 + 32] + data[head:]))
        out.append(("tokenizer kind", data[:11 + 36] + b"byte_bpx" + data[11 + 44:]))
    else:
        out.append(("v3 magic below vocabulary 1024", b"NPRTCKPTV3\n" + data[11:]))
    return out


@needs_ref
@pytest.mark.parametrize("dims,tok", CONFIGS, ids=["V32_L2", "V40_L3", "V1024_L1_v3"])
def test_reader_rejections_match_the_reference_codes(dims, tok, ref, tmp_path):
    cfg, oc = _cfgs(dims)
    n = cfg.parameter_count()
    p, m, v = _state(n, 13)
    kind, hsh = tok if tok else (None, None)
    data = ck.encode(cfg, 99, 12, p, m, v, kind, hsh)
    path = str(tmp_path / "case.ckpt")
    for label, bad in _mutations(data, dims, tok):
        open(path, "wb").write(bad)
        ok, ref_err, *_ = ref.load(path, oc, 99, n, hsh)
        assert not ok, label
        with pytest.raises(ck.CheckpointError) as e:
            ck.decode(cfg, bad, 99, hsh)
        assert str(e.value) == ref_err, (label, str(e.value), ref_err)


@needs_ref
def test_identity_mismatches_match_the_reference_codes(ref, tmp_path):
    """Seed, configuration (tokens, dimension, FFN, layers) and tokenizer
    hash mismatches (nicopedia_resume_test.cpp:615-690)."""
    dims = (1024, 8, 16, 16, 1, 2)
    cfg, oc = _cfgs(dims)
    n = cfg.parameter_count()
    data = ck.encode(cfg, 5, 3, *_state(n, 14), "byte_bpe", HASH)
    path = str(tmp_path / "id.ckpt")
    open(path, "wb").write(data)
    cases = [("seed", dims, 6, HASH), ("tokens", (1024, 16, 16, 16, 1, 2), 5, HASH),
             ("dimension", (1024, 8, 32, 16, 1, 2), 5, HASH), ("ffn", (1024, 8, 16, 32, 1, 2), 5, HASH),
             ("layers", (1024, 8, 16, 16, 2, 2), 5, HASH), ("tokenizer hash", dims, 5, "sha256:" + "f" * 64),
             ("no tokenizer hash", dims, 5, None)]
    for label, d, seed, h in cases:
        c2, o2 = _cfgs(d)
        ok, ref_err, *_ = ref.load(path, o2, seed, c2.parameter_count(), h)
        assert not ok, label
        with pytest.raises(ck.CheckpointError) as e:
            ck.decode(c2, data, seed, h)
        assert str(e.value) == ref_err, (label, str(e.value), ref_err)


@needs_ref
def test_v1_and_nonfinite_files_decode_as_the_reference_reports(ref, tmp_path):
    """A V1 file (parameters only) decodes with has_adam false; non-finite
    values decode with finite false (the reference's generation loader)."""
    dims = (32, 4, 8, 16, 2, 2)
    cfg, oc = _cfgs(dims)
    n = cfg.parameter_count()
    p, m, v = _state(n, 15)
    data = ck.encode(cfg, 1, 4, p, m, v)
    reg_bytes = (len(data) - 43) // 3
    v1 = b"NPRTCKPTV1\n" + data[11:43 + reg_bytes]
    path = str(tmp_path / "v1.ckpt")
    open(path, "wb").write(v1)
    ok, err, rinfo, *_ = ref.load(path, oc, 1, n)
    assert ok, err
    info, p2, m2, v2 = ck.decode(cfg, v1, 1)
    assert not info.has_adam and not rinfo["has_adam"] and m2 is None and np.array_equal(p2, p)
    # a NaN stored in the second-moment registry
    bad = bytearray(data)
    bad[-4:] = struct.pack("<f", float("nan"))
    open(path, "wb").write(bytes(bad))
    ok, err, rinfo, *_ = ref.load(path, oc, 1, n)
    assert ok and not rinfo["finite"]
    info, *_ = ck.decode(cfg, bytes(bad), 1)
    assert not info.finite


@needs_ref
def test_writers_refuse_the_same_states(ref, oracle, tmp_path):
    cfg, oc = _cfgs((32, 4, 8, 16, 2, 2))
    bpe, obpe = _cfgs((1024, 8, 16, 16, 1, 2))
    n, nb = cfg.parameter_count(), bpe.parameter_count()
    p, m, v = _state(n, 16)
    pn = p.copy()
    pn[3] = np.inf
    cases = [(cfg, oc, 0, (p, m, v), None, None), (cfg, oc, 3, (pn, m, v), None, None),
             (cfg, oc, 3, (p, m, v), "byte_bpe", HASH), (bpe, obpe, 3, _state(nb, 1), None, None),
             (bpe, obpe, 3, _state(nb, 1), "byte_bpe", "sha256:short")]
    path = str(tmp_path / "refused.ckpt")
    for c, o, step, st, kind, hsh in cases:
        assert not ref.save(path, o, 1, step, *st, kind, hsh)
        with pytest.raises(ValueError):
            oracle.nprt_encode(o, 1, step, *st, kind, hsh)
        with pytest.raises(ck.CheckpointError):
            ck.encode(c, 1, step, *st, kind, hsh)


@needs_ref
def test_training_order_and_names_match_the_reference(ref, oracle):
    for records, steps, batch in ((1000, 5, 4), (7, 30, 3), (123457, 2, 512)):
        want = ref.training_order(records, steps, batch)
        assert np.array_equal(ck.training_order(records, steps, batch), want)
        assert np.array_equal(oracle.nprt_training_order(records, steps, batch), want)
    for args in ((20260710, 4, 256, 256, 1024, 12), (7, 2, 32, 32, 32, 999999), (1, 1, 64, 48, 48, 5)):
        assert ck.checkpoint_name(*args) == ref.checkpoint_name(*args)


def test_learned_position_registry_round_trip(oracle):
    """The extension entry position_embedding follows token_embedding; the
    oracle writer and the product agree and the product decodes it."""
    cfg, oc = _cfgs((64, 16, 32, 64, 2, 4), learned=True)
    n = cfg.parameter_count()
    p, m, v = _state(n, 17)
    data = ck.encode(cfg, 3, 8, p, m, v)
    assert data == oracle.nprt_encode(oc, 3, 8, p, m, v)
    i = data.index(b"token_embedding")
    j = data.index(b"position_embedding")
    assert i < j < data.index(b"layer_000.norm1_gamma")
    info, p2, m2, v2 = ck.decode(cfg, data, 3)
    assert info.parameter_hash == oracle.nprt_parameter_hash(oc, p)
    assert np.array_equal(p2, p) and np.array_equal(m2, m) and np.array_equal(v2, v)
    # a reference-layout reader of the same dims rejects the extra entry
    plain, _ = _cfgs((64, 16, 32, 64, 2, 4))
    with pytest.raises(ck.CheckpointError, match="NPRT_CKPT_REGISTRY_COUNT_MISMATCH"):
        ck.decode(plain, data, 3)


def test_size_cap_and_empty_input():
    cfg, _ = _cfgs((32, 4, 8, 16, 2, 2))
    with pytest.raises(ck.CheckpointError, match="NPRT_CKPT_SIZE_INVALID"):
        ck.decode(cfg, bytes(64 * 1024 * 1024 + 1), 1)
    with pytest.raises(ck.CheckpointError, match="NPRT_CKPT_MAGIC"):
        ck.decode(cfg, b"", 1)
