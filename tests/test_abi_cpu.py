"""The C-ABI library loads, exports every declared symbol, and its host-side logic (block keys,
launch planning) agrees with the oracle — no GPU needed."""

from __future__ import annotations

import ctypes
import json
import re

import numpy as np
import pytest

from conftest import GOLDEN, ROOT

import muzo_oracle as oracle


def _declared_symbols() -> list[str]:
    text = (ROOT / "include" / "muzo_b200.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(muzo_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(str(ROOT / "muzo-clip_b200" / "muzo_clip_b200" / "libmuzo_b200.so"))
    declared = _declared_symbols()
    assert len(declared) >= 15
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing


def test_python_binding_covers_header():
    from muzo_clip_b200 import _lib

    assert set(_declared_symbols()) == set(_lib.EXPORTED)
    assert _lib.lib.muzo_abi_version() == 2


def _header_constants() -> dict[str, int]:
    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "muzo_b200.h").read_text(), flags=re.S)
    found = dict(re.findall(r"\b(MUZO_[A-Z0-9_]+)\s*=\s*(\d+)", text))
    found.update(re.findall(r"#define\s+(MUZO_[A-Z0-9_]+)\s+(\d+)", text))
    return {k[len("MUZO_"):]: int(v) for k, v in found.items()}


def test_python_constants_match_header():
    """Every enum value and size the binding hard-codes equals the header's."""
    from muzo_clip_b200 import _lib

    consts = _header_constants()
    assert len(consts) >= 30
    checked = 0
    for name, value in consts.items():
        if name in ("ABI_VERSION", "NOALLOC_MAX_BLOCKS"):
            continue
        assert getattr(_lib, name) == value, name
        checked += 1
    assert checked == len(consts) - 2
    assert _lib.lib.muzo_abi_version() == consts["ABI_VERSION"]
    assert _lib.SEGMENT_DTYPE.itemsize == 64


def test_hash_known_answers_native_and_python():
    from muzo_clip_b200 import _lib
    from muzo_clip_b200.prng import hash64_seed

    cases = json.loads((GOLDEN / "hash_kat.json").read_text())
    assert cases
    for c in cases:
        key = c["key"]
        assert hash64_seed(c["seed"], c["name"], tuple(c["shape"]), c["block"]) == key
        assert oracle.hash64_seed(c["seed"], c["name"], tuple(c["shape"]), c["block"]) == key
        assert _lib.hash64_seed_native(c["seed"], c["name"], tuple(c["shape"]), c["block"]) == key


@pytest.mark.parametrize("numel", [1, 255, 256, 1000, 303104, 303105, 1 << 22, (1 << 29) + 1000, (1 << 31) + 64,
                                   (1 << 33) + 12345])
@pytest.mark.parametrize("dist", [0, 1])
def test_native_planner_matches_oracle(numel, dist):
    from muzo_clip_b200 import _lib

    segs, total = _lib.plan_segments([numel], [4096], [8192], dist, 148, 2048)
    launches = oracle.noise_launches(numel, 4 if dist == 0 else 1, 148, 2048)
    assert len(segs) == len(launches)
    items = 0
    for s, l in zip(segs, launches):
        assert int(s["elem_start"]) == l.start
        assert int(s["numel"]) == l.count
        assert int(s["threads"]) == l.threads
        assert int(s["philox_offset"]) == l.offset
        assert int(s["item_begin"]) == items
        assert int(s["param"]) == 4096 and int(s["out"]) == 8192
        trips = (l.count - 1) // (l.threads * 4) + 1
        n = trips * (l.threads // 8)
        items += (n + _lib.ITEMS_PER_CTA - 1) // _lib.ITEMS_PER_CTA * _lib.ITEMS_PER_CTA
    assert total == items


def test_linear_planner():
    from muzo_clip_b200 import _lib

    segs, total = _lib.plan_linear([10, 8192 * 1024 + 3, 1], [1, 2, 3], [4, 5, 6])
    assert [int(s["numel"]) for s in segs] == [10, 8192 * 1024 + 3, 1]
    assert [int(s["block_index"]) for s in segs] == [0, 1, 2]
    per = [(n + 7) // 8 for n in (10, 8192 * 1024 + 3, 1)]
    per = [(p + 1023) // 1024 * 1024 for p in per]
    assert [int(s["item_begin"]) for s in segs] == [0, per[0], per[0] + per[1]]
    assert total == sum(per)


def test_status_strings_and_bad_args():
    from muzo_clip_b200 import _lib

    assert _lib.lib.muzo_status_string(0) == b"ok"
    assert _lib.lib.muzo_status_string(3).startswith(b"pointer")
    # null tables are rejected before anything touches a device
    assert _lib.lib.muzo_perturb_segments(None, 1, 1024, None, 1, 0, 1.0, None) == 1
    assert _lib.lib.muzo_ns_gemm(None, 8, 0, 0, None, 8, 0, 0, None, 8, 0, None, 0, 0.0, 0.0, 8, 8, 8, 1, 0, None, None, None, None, None) == 1
    # unaligned leading dimension
    assert _lib.lib.muzo_ns_gemm(16, 12, 0, 0, 16, 8, 0, 0, 16, 8, 0, None, 0, 0.0, 0.0, 8, 8, 8, 1, 0, None, None, None, None, None) == 3


# A fake, never-dereferenced device address: every call below is rejected by the library's host
# checks before anything is launched (safe with or without a GPU).
_P = 256


@pytest.mark.parametrize("call, expected", [
    # noise and perturbation: table, keys, enums, item counts
    (lambda L: L.muzo_fill_noise(None, 1, 1024, 1, 0, 1, None), 1),
    (lambda L: L.muzo_fill_noise(_P, 1, 1000, 1, 0, 1, None), 1),          # not whole CTAs
    (lambda L: L.muzo_fill_noise(_P, 1, 1024, 1, 0, 9, None), 2),          # dtype
    (lambda L: L.muzo_fill_noise(_P, 1, 1024, 1, 7, 1, None), 1),          # distribution
    (lambda L: L.muzo_perturb_segments(_P, 1, 1024, None, 1, 0, 1.0, None), 1),
    (lambda L: L.muzo_perturb_segments(_P, 1, 1024, _P, 1, 5, 1.0, None), 1),
    (lambda L: L.muzo_perturb_segments(_P, 1, 1024, _P, 9, 0, 1.0, None), 2),
    (lambda L: L.muzo_perturb_segments(None, 0, 0, None, 9, 0, 1.0, None), 0),   # empty: no-op
    (lambda L: L.muzo_perturb_segments_keep_noise(None, 1, 1024, _P, 1, 1.0, None), 1),
    (lambda L: L.muzo_perturb_segments_keep_noise(_P, 1, 1024, None, 1, 1.0, None), 1),
    (lambda L: L.muzo_perturb_segments_keep_noise(_P, 1, 1024, _P, 9, 1.0, None), 2),
    (lambda L: L.muzo_perturb_kept_noise(None, 1, 1024, 1, 1.0, None), 1),
    (lambda L: L.muzo_perturb_kept_noise(_P, 1, 1000, 1, 1.0, None), 1),
    (lambda L: L.muzo_perturb_kept_noise(_P, 1, 1024, 9, 1.0, None), 2),
    (lambda L: L.muzo_perturb_kept_noise(None, 0, 0, 9, 1.0, None), 0),          # empty: no-op
    (lambda L: L.muzo_rebuild_segments_kept(None, 1, 1024, _P, _P, 8, 1, 1, 1.0, _P, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments_kept(_P, 1, 1024, _P, _P, 0, 1, 1, 1.0, _P, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments_kept(_P, 1, 1024, _P, None, 8, 1, 1, 1.0, _P, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments_kept(_P, 1, 1024, _P, _P, 8, 9, 1, 1.0, _P, _P, 0, None), 2),
    (lambda L: L.muzo_rebuild_segments_history(_P, 1, 1024, _P, _P, None, 8, 1, 1, 1.0, _P, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments_history(_P, 1, 1024, _P, _P, _P, 0, 1, 1, 1.0, _P, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments_history(_P, 1, 1000, _P, _P, _P, 8, 1, 1, 1.0, _P, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments_history(_P, 1, 1024, _P, _P, _P, 8, 7, 1, 1.0, _P, _P, 0, None), 2),
    (lambda L: L.muzo_rebuild_kept_linear(_P, 1, 1024, _P, None, 8, 1, 1, 1.0, _P, _P, None), 1),
    (lambda L: L.muzo_rebuild_kept_linear(_P, 1, 1024, _P, _P, 8, 1, 1, 1.0, None, _P, None), 1),
    (lambda L: L.muzo_rebuild_kept_linear(_P, 1, 1024, _P, _P, 8, 5, 1, 1.0, _P, _P, None), 2),
    (lambda L: L.muzo_rebuild_segments(_P, 1, 1024, _P, _P, 0, 0, 1, 1, 1.0, _P, _P, 0, None), 1),  # horizon
    (lambda L: L.muzo_rebuild_segments(_P, 1, 1024, _P, _P, 8, 0, 1, 1, 1.0, None, _P, 0, None), 1),
    (lambda L: L.muzo_rebuild_segments(_P, 1, 1024, _P, _P, 8, 0, 9, 1, 1.0, _P, _P, 0, None), 2),
    # element-wise step kernels
    (lambda L: L.muzo_ns_prepare(_P, 1, 1024, 1, None, _P, None), 1),
    (lambda L: L.muzo_ns_prepare(_P, 1, 1024, 9, _P, _P, None), 2),
    (lambda L: L.muzo_ns_normalize(None, 1, 1024, _P, _P, None), 1),
    (lambda L: L.muzo_ns_normalize(_P, 1, 1024, _P, None, None), 1),
    (lambda L: L.muzo_update_sumsq(_P, 1, 1024, None, _P, _P, None), 1),
    (lambda L: L.muzo_apply_update(_P, 1, 1024, 1, _P, 1e-3, 0.01, 1, 1.0, _P, _P, None, None), 1),
    (lambda L: L.muzo_apply_update(_P, 1, 1024, 9, _P, 1e-3, 0.01, 1, 1.0, _P, _P, _P, None), 2),
    (lambda L: L.muzo_ns_normalize_noalloc(None, None, None, 65, 1, _P, None), 1),
    (lambda L: L.muzo_ns_normalize_noalloc((ctypes.c_void_p * 65)(), (ctypes.c_void_p * 65)(),
                                           (ctypes.c_int64 * 65)(), 65, 1, _P, None), 5),  # capacity
    (lambda L: L.muzo_ns_normalize_noalloc((ctypes.c_void_p * 1)(), (ctypes.c_void_p * 1)(),
                                           (ctypes.c_int64 * 1)(), 1, 9, _P, None), 2),
    # Newton-Schulz GEMM: epilogue operand, epilogue code, symmetric shapes, leading dimensions
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, None, 1, 1.0, 1.0, 8, 8, 8, 1, 0, None, None, None, None, None), 1),
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, _P, 3, 1.0, 1.0, 8, 8, 8, 1, 0, None, None, None, None, None), 1),
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 16, 0, None, 0, 0.0, 0.0, 8, 16, 8, 1, 1, None, None, None, None, None), 1),
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, _P, 2, 1.0, 0.0, 8, 8, 8, 1, 1, None, None, None, None, None), 1),
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, None, 0, 0.0, 0.0, 8, 8, 16, 1, 0, None, None, None, None, None), 1),
    (lambda L: L.muzo_ns_gemm(_P + 8, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, None, 0, 0.0, 0.0, 8, 8, 8, 1, 0, None, None, None, None, None), 3),
    # weight exchange: null arguments and negative counts are rejected before any CUDA call
    (lambda L: L.muzo_ipc_export(None, _P, _P, None), 1),
    (lambda L: L.muzo_ipc_export(_P, None, _P, None), 1),
    (lambda L: L.muzo_ipc_import(None, _P), 1),
    (lambda L: L.muzo_ipc_close(None), 1),
    (lambda L: L.muzo_push_blocks(None, None, None, -1, None), 1),
    (lambda L: L.muzo_push_blocks(None, _P, _P, 2, None), 1),
    (lambda L: L.muzo_push_blocks(None, None, None, 0, None), 0),
    # sums of squares only with the update epilogue, and then with scales and flags
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, _P, 1, 1.0, 1.0, 8, 8, 8, 1, 0, _P, _P, _P, None, None), 1),
    (lambda L: L.muzo_ns_gemm(_P, 8, 0, 0, _P, 8, 0, 0, _P, 8, 0, _P, 2, 1.0, 0.0, 8, 8, 8, 1, 0, _P, None, _P, None, None), 1),
    # QK-Clip
    (lambda L: L.muzo_qk_max(None, _P, 1, 1, 8, 8, 16, 16, 128, 0, 0, 0, 0, 0, 0, 1, 1.0, _P, _P, None), 1),
    (lambda L: L.muzo_qk_max(_P, _P, 1, 1, 8, 3, 16, 16, 128, 0, 0, 0, 0, 0, 0, 1, 1.0, _P, _P, None), 1),  # GQA
    (lambda L: L.muzo_qk_max(_P, _P, 9, 1, 8, 8, 16, 16, 128, 0, 0, 0, 0, 0, 0, 1, 1.0, _P, _P, None), 2),
    (lambda L: L.muzo_qk_max_ranges(_P, _P, 1, 1, 8, 8, 16, 16, 128, 0, 0, 0, 0, 0, 0, 1, _P, None, 1.0, _P, _P, None), 1),
    (lambda L: L.muzo_qk_max_ranges(_P, _P, 1, 1, 8, 8, 16, 16, 128, 0, 0, 0, 0, 0, 0, 1, None, _P, 1.0, _P, _P, None), 1),
    (lambda L: L.muzo_qk_max_ranges(_P, _P, 9, 1, 8, 8, 16, 16, 128, 0, 0, 0, 0, 0, 0, 1, _P, _P, 1.0, _P, _P, None), 2),
    (lambda L: L.muzo_logits_head_max(_P, 1, 1, 70000, 4, 4, 0, 0, 0, 0, _P, _P, None), 1),
    (lambda L: L.muzo_logits_head_max(_P, 9, 1, 8, 4, 4, 0, 0, 0, 0, _P, _P, None), 2),
    (lambda L: L.muzo_max_merge(_P, _P, None, -1, None), 1),
    (lambda L: L.muzo_max_merge(_P, _P, None, 0, None), 0),                 # empty: no-op
    (lambda L: L.muzo_qk_scale_rows(None, 1, 2, 2, 2, _P, _P, None), 1),
    (lambda L: L.muzo_qk_scale_rows(_P, 1, 2, 2, 2, _P, None, None), 1),
])
def test_entry_points_reject_bad_arguments_before_any_launch(call, expected):
    from muzo_clip_b200 import _lib

    assert call(_lib.lib) == expected


def test_segment_layout_matches_header():
    """muzo_segment's fields (order, names, sizes) in the header equal the binding's dtype."""
    from muzo_clip_b200 import _lib

    text = re.sub(r"/\*.*?\*/", "", (ROOT / "include" / "muzo_b200.h").read_text(), flags=re.S)
    body = re.search(r"typedef struct muzo_segment \{(.*?)\} muzo_segment;", text, flags=re.S).group(1)
    fields = re.findall(r"(void\*|u?int\d+_t)\s+(\w+);", body)
    size = {"void*": 8, "int64_t": 8, "uint64_t": 8, "int32_t": 4, "uint32_t": 4}
    assert [name for _, name in fields] == list(_lib.SEGMENT_DTYPE.names)
    assert [size[t] for t, _ in fields] == [_lib.SEGMENT_DTYPE[n].itemsize for n in _lib.SEGMENT_DTYPE.names]
    assert sum(size[t] for t, _ in fields) == _lib.SEGMENT_DTYPE.itemsize == 64
