"""The C ABI: the library loads without a GPU and exports exactly what include/pkv.h declares."""

from __future__ import annotations

import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "pkv.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"^PKV_API\s+[\w\s\*]+?\b(pkv_\w+)\s*\(", text, flags=re.M))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for required in ("pkv_kv_append", "pkv_decode_attention", "pkv_prefill_attention", "pkv_build_decode_metadata",
                     "pkv_build_prefill_metadata", "pkv_copy_blocks", "pkv_bm_allocate", "pkv_bm_free",
                     "pkv_bm_register_prefix", "pkv_bm_ensure_capacity", "pkv_rope_append",
                     "pkv_lm_head_argmax", "pkv_lm_head_argmax_workspace_bytes"):
        assert required in names
    assert len(names) >= 30


def test_library_loads_and_exports_every_declared_symbol():
    from mini_inference_b200 import _lib

    lib = ctypes.CDLL(str(_lib.LIB_PATH))
    missing = [n for n in sorted(declared_functions()) if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert exported == declared_functions(), exported ^ declared_functions()


def test_python_binding_covers_the_header():
    from mini_inference_b200 import _lib

    assert set(_lib.SIGNATURES) == declared_functions()


def test_host_calls_work_without_a_gpu():
    from mini_inference_b200 import _lib

    assert _lib.lib.pkv_version() == 0x000100
    assert _lib.status_name(_lib.PKV_ERR_NO_BLOCKS) == "not enough free KV cache blocks"
    # Shape validation happens before any CUDA call.
    assert _lib.lib.pkv_decode_workspace_bytes(64, 2, 129, 16, 64, 14) > 0
    assert _lib.lib.pkv_decode_workspace_bytes(64, 2, 129, 8, 64, 14) == 0  # block size 8 is not built
    pool = _lib.PkvPool(None, None, 1, 4, 2, 16, 96, _lib.PKV_F16)
    tables = _lib.PkvTables(None, 0, 0, 0, None)
    assert _lib.lib.pkv_decode_attention(ctypes.byref(pool), 0, ctypes.byref(tables), 1, 14, None, 0, 0, None, 0, 0,
                                         None, None, 0, 0, None, None, 1.0, 0, None, 0, None, None) \
        == _lib.PKV_ERR_INVALID_ARGUMENT


def test_import_fails_loudly_without_the_library(tmp_path, monkeypatch):
    """Without libpkv.so the package cannot be imported: there is no silent fallback."""
    import importlib.util
    import sys

    src = (ROOT / "mini_inference_b200" / "_lib.py").read_text()
    fake = tmp_path / "_lib.py"
    fake.write_text(src)
    spec = importlib.util.spec_from_file_location("pkv_lib_without_so", fake)
    mod = importlib.util.module_from_spec(spec)
    with pytest.raises(ImportError, match="not built"):
        spec.loader.exec_module(mod)
    sys.modules.pop("pkv_lib_without_so", None)


def test_lm_head_argmax_validates_on_the_host():
    from mini_inference_b200 import _lib

    L = _lib.lib
    assert L.pkv_lm_head_argmax_workspace_bytes(64) == 8 + 8 * 64
    # Null pointers, then shapes the kernel does not take (checked before any CUDA call).
    assert L.pkv_lm_head_argmax(None, 896, 4, None, 896, 1000, 896, _lib.PKV_F16, None, None, None, 0, 0, None,
                                None) == _lib.PKV_ERR_INVALID_ARGUMENT
    fake = ctypes.c_void_p(1 << 20)  # aligned, never dereferenced: validation returns first
    args = dict(hidden_stride=896, batch=4, weight_stride=896, vocab=1000, hidden=896, dtype=_lib.PKV_F16, ws=4096)

    def call(**kw):
        a = {**args, **kw}
        return L.pkv_lm_head_argmax(fake, a["hidden_stride"], a["batch"], fake, a["weight_stride"], a["vocab"],
                                    a["hidden"], a["dtype"], fake, None, fake, a["ws"], 0, None, None)

    assert call(hidden=96, hidden_stride=96, weight_stride=96) == _lib.PKV_ERR_UNSUPPORTED  # not a multiple of 64
    assert call(batch=257, ws=1 << 16) == _lib.PKV_ERR_UNSUPPORTED
    assert call(dtype=7) == _lib.PKV_ERR_UNSUPPORTED
    assert call(hidden_stride=900) == _lib.PKV_ERR_INVALID_ARGUMENT  # rows not 16-byte aligned
    assert call(ws=16) == _lib.PKV_ERR_WORKSPACE
    assert call(batch=0) == _lib.PKV_OK


def test_static_scratch_size_matches_the_header():
    from mini_inference_b200 import _lib

    m = re.search(r"#define\s+PKV_DECODE_STATIC_SCRATCH_BYTES\s+\(([^)]*)\)", HEADER.read_text())
    assert m, "PKV_DECODE_STATIC_SCRATCH_BYTES is not defined in pkv.h"
    assert eval(m.group(1), {"__builtins__": {}}) == _lib.PKV_DECODE_STATIC_SCRATCH_BYTES


def test_workspace_reset_validates_before_any_cuda_call():
    from mini_inference_b200 import _lib

    assert _lib.lib.pkv_decode_reset_workspace(None, 1 << 20, None) == _lib.PKV_ERR_INVALID_ARGUMENT
    assert _lib.lib.pkv_decode_static_scratch(None, None, None) == _lib.PKV_ERR_INVALID_ARGUMENT


def test_layer_ops_validate_before_any_cuda_call():
    from mini_inference_b200 import _lib

    L, bad, uns = _lib.lib, _lib.PKV_ERR_INVALID_ARGUMENT, _lib.PKV_ERR_UNSUPPORTED
    fake = 1 << 20  # never dereferenced: every case below is refused on the host
    assert L.pkv_add_rms_norm(_lib.PKV_F16, None, 896, None, 0, None, 0, fake, fake, 896, 4, 896, 1e-6, None) == bad
    assert L.pkv_add_rms_norm(_lib.PKV_F16, fake, 64, None, 0, None, 0, fake, fake, 896, 4, 896, 1e-6, None) == bad
    assert L.pkv_add_rms_norm(_lib.PKV_F16, fake, 896, None, 0, None, 0, fake, fake, 896, 4, 896, -1.0, None) == bad
    assert L.pkv_add_rms_norm(99, fake, 896, None, 0, None, 0, fake, fake, 896, 4, 896, 1e-6, None) == uns
    assert L.pkv_add_rms_norm(_lib.PKV_F16, fake, 896, None, 0, None, 0, fake, fake, 896, 0, 896, 1e-6, None) == 0
    assert L.pkv_silu_mul(_lib.PKV_F16, None, 9728, fake, 4864, 4, 4864, None) == bad
    assert L.pkv_silu_mul(_lib.PKV_F16, fake, 4864, fake, 4864, 4, 4864, None) == bad  # gate_up row too short
    assert L.pkv_silu_mul(99, fake, 9728, fake, 4864, 4, 4864, None) == uns
    assert L.pkv_silu_mul(_lib.PKV_BF16, fake, 9728, fake, 4864, 0, 4864, None) == 0


def test_norm_partials_validate_before_any_cuda_call():
    from mini_inference_b200 import _lib

    L, bad, uns = _lib.lib, _lib.PKV_ERR_INVALID_ARGUMENT, _lib.PKV_ERR_UNSUPPORTED
    fake = 1 << 20  # never dereferenced: every case below is refused (or empty) on the host
    def call(dtype=_lib.PKV_F16, row_stride=896, splits=4, split_stride=4 * 896, rows=4, hidden=896):
        return L.pkv_add_rms_norm_partials(dtype, fake, row_stride, splits, split_stride, None, 0, None, 0, fake,
                                           fake, 896, rows, hidden, 1e-6, None)

    assert call(splits=0) == bad
    assert call(row_stride=64) == bad
    assert call(split_stride=896) == bad  # slices would overlap
    assert call(dtype=99) == uns
    assert call(rows=0, split_stride=0) == 0
