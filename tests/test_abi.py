"""The C ABI without a GPU: libfa_attn.so loads, exports every entry point include/fa_attn.h
declares, and its host-side logic (rotary tables, the seeded generator, argument checks that
stand in for the reference's panics) agrees with the reference and the oracle."""
import ctypes as C
import json
import os
import re
import subprocess

import numpy as np
import pytest

import fusor_attn as fa
import oracle

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "fa_attn.h")
GOLDEN = os.path.join(ROOT, "tests", "golden")


def declared_entry_points():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"^(?:int|const char\*)\s+(fa_\w+)\(", text, re.M)))


def test_every_declared_entry_point_is_exported():
    names = declared_entry_points()
    assert len(names) >= 19
    out = subprocess.run(["nm", "-D", "--defined-only", fa.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (fa_\w+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    lib = fa.lib()
    for n in names:
        assert getattr(lib, n) is not None
    assert set(names) == set(fa.SIGNATURES)


def test_library_has_no_cuda_runtime_or_oracle_dependency():
    out = subprocess.run(["ldd", fa.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcudart" not in out
    assert "oracle" not in out
    syms = subprocess.run(["nm", "-D", fa.LIB_PATH], capture_output=True, text=True).stdout
    assert "oracle_" not in syms


def test_rotary_angles_are_the_reference_literals():
    with open(os.path.join(GOLDEN, "reference_kats.json")) as f:
        kats = json.load(f)["rotary"]
    kinds = {"axes": fa.ROT_AXES, "linear": fa.ROT_LINEAR}
    for case in kats:
        rot = fa.Rotation(kinds[case["rotation"]], tuple(case["params"]), case["base"],
                          case["spatial_scale"])
        got = fa.rotary_angles(rot, case["head_dim"], [fa.Position(*case["position"])])[0]
        want = np.array(case["want_cos"] + case["want_sin"], np.float32)
        assert np.abs(got - want).max() < case["tolerance"], case["test"]


@pytest.mark.parametrize("kind,params", [
    (fa.ROT_SEQUENCE, (0, 0, 0)), (fa.ROT_LINEAR, (8, 0, 0)), (fa.ROT_PARTIAL, (5, 0, 0)),
    (fa.ROT_MULTIMODAL, (16, 8, 8)), (fa.ROT_AXES, (8, 12, 12)),
    (fa.ROT_MULTIMODAL_INTERLEAVED, (0, 6, 6)), (fa.ROT_GRID, (0, 0, 0))])
def test_rotary_tables_bit_equal_the_oracle(kind, params):
    d = 64
    positions = [fa.Position(p, (p * 7) % 31, (p * 13) % 29) for p in range(0, 3000, 97)]
    got = fa.rotary_angles(fa.Rotation(kind, params, 1e6), d, positions)
    for row, p in zip(got, positions):
        c, s = oracle.rotary_angles(kind, 1e6, d, (p.temporal, p.height, p.width), params)
        assert (row[: d // 2].view(np.uint32) == c.view(np.uint32)).all()
        assert (row[d // 2:].view(np.uint32) == s.view(np.uint32)).all()


def test_rng_is_deterministic_and_standard_normal():
    a = fa.rng_normal(7, 200001)
    b = fa.rng_normal(7, 200001)
    assert (a.view(np.uint32) == b.view(np.uint32)).all()
    assert abs(a.mean()) < 0.01 and abs(a.std() - 1.0) < 0.01
    assert not np.array_equal(a[:1000], fa.rng_normal(8, 1000))


def test_rng_matches_a_python_restatement_of_rng_rs():
    # crates/kernels/src/rng.rs:10-52, restated independently in Python for a few values.
    m = (1 << 64) - 1
    mixed = 42

    def nxt_seed():
        nonlocal mixed
        mixed = (mixed + 0x9E3779B97F4A7C15) & m
        z = mixed
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & m
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & m
        return z ^ (z >> 31)

    st = [nxt_seed() for _ in range(4)]

    def rotl(x, k):
        return ((x << k) | (x >> (64 - k))) & m

    def nxt():
        res = (rotl((st[1] * 5) & m, 7) * 9) & m
        t = (st[1] << 17) & m
        st[2] ^= st[0]; st[3] ^= st[1]; st[1] ^= st[2]; st[0] ^= st[3]; st[2] ^= t
        st[3] = rotl(st[3], 45)
        return res

    want = []
    for _ in range(5):
        u1 = ((nxt() >> 11) + 1) / float(1 << 53)
        u2 = ((nxt() >> 11) + 1) / float(1 << 53)
        r = np.sqrt(-2.0 * np.log(u1))
        want += [np.float32(r * np.cos(2 * np.pi * u2)), np.float32(r * np.sin(2 * np.pi * u2))]
    got = fa.rng_normal(42, 10)
    assert np.allclose(got, np.array(want, np.float32), rtol=0, atol=1e-6)


def test_shape_errors_are_status_codes_not_panics():
    h = C.c_void_p()
    rc = fa.lib().fa_kvcache_create(1, 14, 4, 64, 16, fa.F32, 0, C.byref(h))
    assert rc == fa.ERR_SHAPE
    assert b"14 heads over 4 KV heads" in fa.lib().fa_last_error()
    # head dims off the kernels' 16-byte vectors, or past 256: no kernel (52 f32 and 80 bf16 have
    # one, the next wider kernel's; 52 bf16 is not a whole number of 8-element vectors)
    for d, dtype in ((50, fa.F32), (52, fa.BF16), (260, fa.F32), (24, fa.F32)):
        assert fa.lib().fa_kvcache_create(1, 4, 2, d, 16, dtype, 0, C.byref(h)) == fa.ERR_UNSUPPORTED
    assert fa.lib().fa_kvcache_create(1, 4, 2, 64, 0, fa.F32, 0, C.byref(h)) == fa.ERR_ARG
    assert fa.lib().fa_kvcache_create(1, 4, 2, 64, 8, 7, 0, C.byref(h)) == fa.ERR_ARG
    assert fa.lib().fa_kvcache_create(1, 4, 2, 64, 8, fa.F32, 0, None) == fa.ERR_ARG
    assert fa.lib().fa_attention(None, 0, None, 0, None, None, None, 0, None, 0, None) == fa.ERR_ARG


def test_rotary_argument_errors():
    bad = fa.Rotation(fa.ROT_AXES, (1, 1, 1), 1e4)
    with pytest.raises(fa.FaError):
        fa.rotary_angles(bad, 64, [0])
    with pytest.raises(fa.FaError):
        fa.rotary_angles(fa.Rotation(99), 64, [0])


def test_capabilities():
    flags, dims = fa.capabilities()
    assert flags & 1 and flags & 2 and flags & 8  # f32, bf16, head dims between the powers of two
    assert dims == [16, 32, 64, 128, 256]


def test_peer_exchange_buffer_size_and_arguments():
    """fa_peer_buffer_bytes: a 256-byte header (the step counter), then two halves of world x
    heads x (head_dim + 2) partials, each value a 64-bit word (its step stamp and its f32 bits);
    worlds past the 8 GPUs of a box, and a
    fa_exchange_merge whose buffers are smaller than that, are refused before any launch."""
    lib = fa.lib()
    n = C.c_uint64()
    assert lib.fa_peer_buffer_bytes(8, 16, 128, C.byref(n)) == fa.OK
    assert n.value == 256 + 2 * 8 * 16 * 130 * 8  # 64-bit stamped words
    assert lib.fa_peer_buffer_bytes(9, 16, 128, C.byref(n)) == fa.ERR_ARG
    assert lib.fa_peer_buffer_bytes(0, 16, 128, C.byref(n)) == fa.ERR_ARG
    bufs = (C.c_void_p * 2)(1, 2)
    rc = lib.fa_exchange_merge(bufs, 256, 0, 2, 16, 128, C.c_void_p(16), C.c_void_p(16), None)
    assert rc == fa.ERR_SHAPE
    assert b"exchange buffers" in lib.fa_last_error()
    rc = lib.fa_exchange_merge(bufs, 1 << 20, 2, 2, 16, 128, C.c_void_p(16), C.c_void_p(16), None)
    assert rc == fa.ERR_ARG


def test_batch_host_call_refuses_bad_arguments_before_any_copy():
    """fa_attention_batch_host checks its arguments on the host: no caches or spans, and a batch
    past 1024 sequences, are refused with ERR_ARG before any copy or launch."""
    lib = fa.lib()
    rc = lib.fa_attention_batch_host(None, None, 1, 0, fa.ROPE_NONE, None, None, None, 0, None, 0,
                                     None)
    assert rc == fa.ERR_ARG
    assert b"null caches or spans" in lib.fa_last_error()
    caches = (C.c_void_p * 1)(None)
    spans = (fa._Span * 1)()
    rc = lib.fa_attention_batch_host(caches, spans, 1025, 0, fa.ROPE_NONE, None, None, None, 0,
                                     None, 0, None)
    assert rc == fa.ERR_ARG


def _strip_c_comments(text):
    return re.sub(r"//[^\n]*", "", re.sub(r"/\*.*?\*/", "", text, flags=re.S))


def _rust_ffi_block():
    """The Rust binding's source (rust/fusor-cuda-attn/src/ffi.rs): its structs and its one
    extern block."""
    text = open(os.path.join(ROOT, "rust", "fusor-cuda-attn", "src", "ffi.rs")).read()
    assert text.count('extern "C"') == 1
    return text


def test_rust_binding_declares_every_entry_point_with_its_arity():
    """The Rust extern block a maintainer would add to fusor-ai names each entry point the
    header declares, once, with the header's parameter count (no stale or missing lines)."""
    header = _strip_c_comments(open(HEADER).read())
    want = {}
    for name, params in re.findall(r"\b(fa_\w+)\s*\(([^;{]*?)\)\s*;", header, re.S):
        params = " ".join(params.split())
        want[name] = 0 if params in ("", "void") else params.count(",") + 1
    assert set(want) == set(declared_entry_points())
    got = {}
    for name, params in re.findall(r"pub fn (fa_\w+)\((.*?)\)\s*(?:->[^;]*)?;",
                                   _rust_ffi_block(), re.S):
        assert name not in got, name
        params = " ".join(params.split())
        got[name] = 0 if not params else params.count(":")
    assert got == want


def test_rust_structs_mirror_the_header_structs():
    """Each #[repr(C)] struct of the Rust binding has the C struct's fields in the same order."""
    header = _strip_c_comments(open(HEADER).read())
    c_fields = {}
    for body, name in re.findall(r"typedef struct\s*\w*\s*\{(.*?)\}\s*(\w+)\s*;", header, re.S):
        fields = [re.sub(r"\[.*?\]", "", d).split()[-1].lstrip("*")
                  for d in body.split(";") if d.strip()]
        c_fields[name] = fields
    rust = _rust_ffi_block()
    seen = 0
    for rname, body in re.findall(r"#\[repr\(C\)\] pub struct (\w+) \{(.*?)\}", rust, re.S):
        if rname == "FaKvCache":
            continue
        cname = "fa_" + re.sub(r"(?<!^)([A-Z])", r"_\1", rname[2:]).lower()
        fields = [f.split(":")[0].replace("pub", "").strip() for f in body.split(",") if f.strip()]
        assert fields == c_fields[cname], rname
        seen += 1
    assert seen == len(c_fields)
