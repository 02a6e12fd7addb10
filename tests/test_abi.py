"""The C ABI without a GPU: the library loads, exports every entry point
``include/cevk.h`` declares with the bound signatures, and its host-side
validation (segment scheduling) behaves."""
import ctypes as C
import os
import re

import pytest

from cev_b200 import _lib

HEADER = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "include", "cevk.h")


def declared():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cevk_[a-z0-9_]+)\s*\(", text)))


def test_library_loads_and_exports_every_declared_symbol():
    lib = _lib.lib()
    names = declared()
    assert names, "no declarations parsed"
    for n in names:
        assert hasattr(lib, n), f"{n} not exported"
        assert n in _lib.SIGNATURES, f"{n} not bound in _lib.SIGNATURES"
    assert lib.cevk_version() == 100


def test_binding_arity_matches_header():
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name, (_, args) in _lib.SIGNATURES.items():
        m = re.search(name + r"\s*\(([^)]*)\)", text)
        assert m, name
        params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        assert len(params) == len(args), f"{name}: header has {len(params)} params, binding {len(args)}"


def _segs(rows):
    arr = (_lib.Segment * len(rows))()
    for i, r in enumerate(rows):
        arr[i].q_start, arr[i].q_len, arr[i].prefix_off, arr[i].prefix_len, arr[i].self_off = r
    return arr


def test_schedule_assigns_tiles_per_gqa_group():
    lib = _lib.lib()
    # hq/hkv = 2 -> 64 tokens per tile; a 150-token segment needs 3 tiles.
    arr = _segs([(0, 64, 0, 100, 100), (64, 150, 0, 100, 164), (214, 0, 0, 0, 0), (214, 1, 0, 0, 314)])
    n = C.c_int32()
    assert lib.cevk_attn_schedule(arr, 4, 215, 400, 16, 8, 128, _lib.BF16, C.byref(n)) == 0
    assert [arr[i].tile_start for i in range(4)] == [0, 1, 4, 4]
    assert n.value == 5


@pytest.mark.parametrize("bad", [
    (0, 65, 0, 10, 0),      # query rows past n_tokens
    (0, 10, 390, 20, 0),    # prefix past the arena
    (0, 10, 0, 10, 395),    # own rows past the arena
    (-1, 10, 0, 10, 0),     # negative offset
])
def test_schedule_rejects_out_of_range_segments(bad):
    lib = _lib.lib()
    n = C.c_int32()
    rc = lib.cevk_attn_schedule(_segs([bad]), 1, 64, 400, 16, 8, 128, _lib.BF16, C.byref(n))
    assert rc == _lib.E_RANGE
    assert lib.cevk_last_error().decode()


def test_schedule_rejects_bad_gqa():
    lib = _lib.lib()
    n = C.c_int32()
    assert lib.cevk_attn_schedule(_segs([(0, 1, 0, 0, 0)]), 1, 1, 1, 12, 8, 128, _lib.BF16, C.byref(n)) == _lib.E_SHAPE
    assert lib.cevk_attn_schedule(_segs([(0, 1, 0, 0, 0)]), 1, 1, 1, 24, 8, 128, _lib.BF16, C.byref(n)) == _lib.E_SHAPE


def _plan(rows, n_tok, n_kv, hq, hkv, D, sms=148):
    lib = _lib.lib()
    arr = _segs(rows)
    n = C.c_int32()
    assert lib.cevk_attn_schedule(arr, len(rows), n_tok, n_kv, hq, hkv, D, _lib.BF16, C.byref(n)) == 0
    ns, nb = C.c_int32(), C.c_int64()
    assert lib.cevk_attn_split_plan(arr, len(rows), n.value, hkv, D, _lib.BF16, sms, C.byref(ns), C.byref(nb)) == 0
    return n.value, ns.value, nb.value


def test_split_plan_fills_the_waves_of_underfilled_calls():
    """A 512-token prefill chunk after a long prefix (cfg5's LFM2 chunk:
    32 Q / 8 KV heads, head_dim 64 -> 16 tiles x 8 KV heads = 128 CTAs on
    148 SMs x 2) splits 9 ways (1152 items fill 97% of four waves; 2 ranges
    would fill 86% of one) after 32768 tokens and 2 ways after 8192; one KV
    head per rank (the 8-way KV-head split) splits 18 ways; a short prefix
    or an already full call does not split; the workspace is one f32 row +
    log-sum-exp per range and row."""
    lib = _lib.lib()
    tiles, ns, nb = _plan([(0, 512, 0, 32768, 32768)], 512, 33280, 32, 8, 64)
    assert (tiles, ns) == (16, 9) and nb == 16 * 8 * 9 * 128 * 65 * 4
    assert _plan([(0, 512, 0, 8192, 8192)], 512, 8704, 32, 8, 64)[1] == 2
    assert nb == lib.cevk_attn_split_workspace_size(tiles, 8, 64, ns)
    assert _plan([(0, 512, 0, 32768, 32768)], 512, 33280, 4, 1, 64)[1] == 18
    assert _plan([(0, 512, 0, 448, 448)], 512, 960, 4, 1, 64)[1] == 1        # 7 prefix blocks: too short
    assert _plan([(0, 512, 0, 4096, 4096)], 512, 4608, 4, 1, 64)[1] == 8     # 64 blocks: ranges of >= 8
    rows = [(i * 64, 64, 0, 2048, 2048 + i * 64) for i in range(64)]
    assert _plan(rows, 4096, 6144, 16, 8, 128)[1] == 1                       # 512 CTAs: already full
    assert _plan([(0, 128, 0, 65536, 65536)], 128, 65664, 16, 4, 256)[1] == 9   # 16 CTAs, one per SM at head_dim 256
    assert lib.cevk_attn_split_workspace_size(16, 8, 64, 1) == 0


def test_static_library_links_into_a_plain_c_program(tmp_path):
    """``libcevk.a`` (the objects plus their device-link object) links with
    the host toolchain alone -- as cargo links it through a build.rs -- and
    defines every entry point the header declares."""
    import shutil
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path.insert(0, os.path.join(root, "rust-cev_b200"))
    import build as cevk_build
    lib_a = cevk_build.build(static=True)
    nm = subprocess.run(["nm", "-g", "--defined-only", lib_a], capture_output=True, text=True, check=True).stdout
    defined = set(re.findall(r"\bT (cevk_[a-z0-9_]+)\b", nm))
    assert set(declared()) <= defined, sorted(set(declared()) - defined)
    if shutil.which("gcc") is None:
        pytest.skip("no gcc")
    src = tmp_path / "main.c"
    src.write_text('#include <stdio.h>\n#include "cevk.h"\n'
                   'int main(void) { printf("%d %zu\\n", cevk_version(), '
                   'cevk_gdn_workspace_size(1, 64, 4, 64, 64)); return 0; }\n')
    exe = tmp_path / "main"
    cuda = "/usr/local/cuda/lib64"
    subprocess.run(["gcc", "-I", os.path.join(root, "include"), str(src), lib_a, "-L" + cuda, "-lcudart", "-lcuda",
                    "-lstdc++", "-lm", "-o", str(exe)], check=True, capture_output=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True,
                         env=dict(os.environ, LD_LIBRARY_PATH=cuda)).stdout.split()
    assert out[0] == "100" and int(out[1]) == _lib.lib().cevk_gdn_workspace_size(1, 64, 4, 64, 64)


def test_rust_bindings_match_the_header():
    """The committed Rust binding crate (rust-cev_b200/rust/cevk-sys) binds
    every entry point of the header with the same arity and the same
    status / dtype constants (there is no Rust toolchain here to compile
    it, so the check is textual)."""
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    rs = open(os.path.join(root, "rust-cev_b200", "rust", "cevk-sys", "src", "lib.rs")).read()
    fns = {n: a for n, a in re.findall(r"pub fn (cevk_[a-z0-9_]+)\s*\(([^)]*)\)", rs, flags=re.S)}
    assert set(fns) == set(declared()), sorted(set(fns) ^ set(declared()))
    text = re.sub(r"/\*.*?\*/", "", open(HEADER).read(), flags=re.S)
    for name, args in fns.items():
        m = re.search(name + r"\s*\(([^)]*)\)", text)
        c_params = [p for p in m.group(1).split(",") if p.strip() and p.strip() != "void"]
        rs_params = [p for p in args.split(",") if p.strip()]
        assert len(rs_params) == len(c_params), f"{name}: rust {len(rs_params)} params, header {len(c_params)}"
    for const, val in re.findall(r"#define (CEVK_[A-Z0-9_]+) \(?(-?\d+)\)?", open(HEADER).read()):
        m = re.search(r"pub const " + const + r": \w+ = (-?\d+)", rs)
        assert m and int(m.group(1)) == int(val), const
