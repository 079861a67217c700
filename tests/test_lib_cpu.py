"""libexpertcache.so on a machine without a GPU: it loads, exports every symbol the
public header declares, and refuses bad arguments with -1 before touching CUDA (the
launcher rules of the reference, kernels/expert_cache.hip:596-598 and :632-634)."""

from __future__ import annotations

import ctypes
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
PKG = ROOT / "vllm-expert-cache_b200"


@pytest.fixture(scope="module")
def h():
    import build_lib  # vllm-expert-cache_b200/build_lib.py
    from vllm_expert_cache import _lib
    build_lib.build()
    return _lib.lib()


def test_exports_every_header_symbol(h):
    import build_lib as b
    want = b.exported_symbols()
    assert set(want) == {"expert_cache_manage", "expert_cache_manage_remap",
                         "expert_cache_manage_ep", "expert_cache_prefetch",
                         "expert_cache_pregate", "expert_cache_gather"} | set(want)
    out = subprocess.run(["nm", "-D", "--defined-only", str(b.OUT)], check=True,
                         capture_output=True, text=True).stdout
    have = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert set(want) <= have
    for name in want:
        assert getattr(h, name) is not None


def test_built_for_sm100a_only():
    import build_lib as b
    assert "arch=compute_100a,code=sm_100a" in " ".join(b.FLAGS)


NULL = ctypes.c_void_p(0)


def manage(h, E=8, S=4, mi=4, policy=0, mk=2):
    return h.expert_cache_manage(NULL, mk, E, S, 8, mi, *([NULL] * 8), policy, 64, NULL)


@pytest.mark.parametrize("kw", [dict(E=0), dict(E=-3), dict(E=32769), dict(S=0),
                                dict(S=1025), dict(mi=-1), dict(mi=1025), dict(policy=2),
                                dict(policy=-1)])
def test_manage_refuses_bad_arguments(h, kw):
    assert manage(h, **kw) == -1


def test_manage_remap_refuses_bad_output(h):
    args = [NULL, 2, 8, 4, 8, 4, *([NULL] * 8), 0, 64]
    assert h.expert_cache_manage_remap(*args, NULL, 4, NULL) == -1
    buf = ctypes.create_string_buffer(64)
    assert h.expert_cache_manage_remap(*args, ctypes.cast(buf, ctypes.c_void_p), 2,
                                       NULL) == -1
    bad = [NULL, 2, 0, 4, 8, 4, *([NULL] * 8), 0, 64]
    assert h.expert_cache_manage_remap(*bad, ctypes.cast(buf, ctypes.c_void_p), 4,
                                       NULL) == -1


def test_manage_ep_refuses_bad_arguments(h):
    buf = ctypes.cast(ctypes.create_string_buffer(64), ctypes.c_void_p)
    state = [NULL] * 8

    def ep(emap=buf, Eg=16, E=8, S=4, out=buf, policy=0):
        return h.expert_cache_manage_ep(NULL, 2, emap, Eg, E, S, 8, 4, *state, policy, 64,
                                        out, NULL)
    assert ep(emap=NULL) == -1
    assert ep(out=NULL) == -1
    assert ep(Eg=0) == -1
    assert ep(E=0) == -1 and ep(S=1025) == -1 and ep(policy=3) == -1


def test_prefetch_refuses_bad_arguments(h):
    def pf(E=8, S=4, mi=4, policy=0):
        return h.expert_cache_prefetch(NULL, 2, E, S, 8, mi, *([NULL] * 8), policy, NULL)
    assert pf(E=0) == -1 and pf(S=0) == -1 and pf(mi=-1) == -1 and pf(policy=2) == -1


@pytest.mark.parametrize("kw", [dict(T=-1), dict(H=0), dict(H=12), dict(H=16392),
                                dict(ldx=8), dict(ldx=20), dict(E=0), dict(E=2049),
                                dict(k=0), dict(k=33), dict(x=8), dict(w=24)])
def test_pregate_refuses_bad_arguments(h, kw):
    a = dict(T=2, ldx=16, H=16, E=8, k=4, x=256, w=512)
    a.update(kw)
    out = ctypes.c_void_p(1024)
    assert h.expert_cache_pregate(ctypes.c_void_p(a["x"]), a["T"], a["ldx"], a["H"],
                                  ctypes.c_void_p(a["w"]), a["E"], a["k"], out, NULL) == -1


def test_pregate_empty_batch_enqueues_nothing(h):
    assert h.expert_cache_pregate(ctypes.c_void_p(256), 0, 16, 16, ctypes.c_void_p(512), 8,
                                  4, ctypes.c_void_p(1024), NULL) == 0


def gather(h, sizes, chunks=16, lanes=64, ptr=256):
    args = []
    for b in sizes:
        args += [ctypes.c_void_p(ptr), ctypes.c_void_p(ptr), ctypes.c_long(b)]
    return h.expert_cache_gather(*args, NULL, NULL, chunks, lanes, NULL)


@pytest.mark.parametrize("sizes", [[16] * 5 + [0], [16] * 5 + [-16], [16, 24, 16, 16, 16, 16]])
def test_gather_refuses_bad_sizes(h, sizes):
    assert gather(h, sizes) == -1


def test_gather_refuses_bad_grid_and_alignment(h):
    assert gather(h, [16] * 6, chunks=0) == -1
    assert gather(h, [16] * 6, lanes=-1) == -1
    assert gather(h, [16] * 6, ptr=8) == -1


def step(h, E=8, S=4, mi=4, policy=0, mk=2, out=True, elem=4, sizes=(16,) * 6, ptr=256,
         chunks=16, lanes=64, sync=512, wait=0):
    buf = ctypes.c_void_p(1024) if out else NULL
    trip = []
    for b in sizes:
        trip += [ctypes.c_void_p(ptr), ctypes.c_void_p(ptr), ctypes.c_long(b)]
    return h.expert_cache_step(NULL, mk, E, S, 8, mi, *([NULL] * 8), policy, 64, buf, elem,
                               *trip, chunks, lanes, ctypes.c_void_p(sync), wait, NULL)


@pytest.mark.parametrize("kw", [dict(E=0), dict(S=0), dict(S=257), dict(mi=1025),
                                dict(policy=2), dict(out=False), dict(elem=2),
                                dict(sizes=(16,) * 5 + (24,)), dict(ptr=8), dict(chunks=0),
                                dict(lanes=-1), dict(sync=0), dict(sync=514), dict(wait=-1),
                                dict(sizes=(1 << 36,) * 6, mi=1024)])
def test_step_refuses_bad_arguments(h, kw):
    # refused before any CUDA call: these return -1 on a machine without a GPU
    assert step(h, **kw) == -1


def test_library_search_order(monkeypatch, tmp_path):
    from vllm_expert_cache import _lib
    fake = tmp_path / "libexpertcache.so"
    fake.write_bytes(b"")
    monkeypatch.setenv("EXPERT_CACHE_LIB", str(fake))
    assert _lib.library_path() == str(fake)
    monkeypatch.setenv("EXPERT_CACHE_LIB", str(tmp_path / "absent.so"))
    assert _lib.library_path().endswith("vllm_expert_cache/libexpertcache.so")


def test_missing_library_is_loud(monkeypatch, tmp_path):
    from vllm_expert_cache import _lib
    monkeypatch.setenv("EXPERT_CACHE_LIB", "")
    monkeypatch.setattr(_lib, "_candidates", lambda: iter([str(tmp_path / "nope.so")]))
    with pytest.raises(FileNotFoundError):
        _lib.library_path()


def test_config_quirks(monkeypatch):
    from vllm_expert_cache.config import settings
    monkeypatch.delenv("EXPERT_CACHE_SLOTS", raising=False)
    monkeypatch.delenv("EXPERT_CACHE_FRACTION", raising=False)
    assert settings.slots_for(128) == 64
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", "0")
    assert settings.slots_for(128) == 1          # 0 clamps to one slot, not "off"
    monkeypatch.setenv("EXPERT_CACHE_SLOTS", "500")
    assert settings.slots_for(128) == 128
    monkeypatch.setenv("EXPERT_CACHE_POLICY", " LRU ")
    assert settings.policy_code == 0
    monkeypatch.setenv("EXPERT_CACHE_POLICY", "fifo")
    assert settings.policy_code == 0             # unknown -> LRU
    monkeypatch.delenv("EXPERT_CACHE_POLICY")
    assert settings.policy == "lfu" and settings.policy_code == 1
    assert settings.decay == 64 and settings.chunks == 16 and settings.lanes == 64
    monkeypatch.setenv("EXPERT_CACHE_DISABLE", "1")
    assert settings.disabled


def test_entry_point_declared():
    text = (PKG / "pyproject.toml").read_text()
    assert '[project.entry-points."vllm.general_plugins"]' in text
    assert 'expert_cache = "vllm_expert_cache:install"' in text


def test_install_respects_disable(monkeypatch):
    import vllm_expert_cache
    monkeypatch.setenv("EXPERT_CACHE_DISABLE", "1")
    vllm_expert_cache.install()   # returns without importing vLLM's loader


def fused(h, E=8, S=4, mi=4, mk=2, bs=16, L=32, NB=2):
    return h.expert_cache_fused(NULL, mk, E, S, 8, mi, *([NULL] * 8), bs, L, NB,
                                *([NULL] * 6), NULL)


@pytest.mark.parametrize("kw", [dict(E=0), dict(E=1025), dict(S=0), dict(S=1025),
                                dict(bs=0), dict(L=0), dict(NB=0), dict(mk=-1),
                                dict(mi=-1), dict(mi=1025)])
def test_fused_refuses_bad_arguments(h, kw):
    import ctypes as C
    P, I = C.c_void_p, C.c_int
    h.expert_cache_fused.restype = I
    h.expert_cache_fused.argtypes = [P] + [I] * 5 + [P] * 8 + [I, I, I] + [P] * 6 + [P]
    assert fused(h, **kw) == -1
