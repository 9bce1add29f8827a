"""The C-ABI library builds, loads and exports every symbol include/ms_engine.h
declares; argument checks that run before any CUDA call behave like the
reference prototype's (scripts/validate_cuda_kernels.py:120-122).  No GPU."""
import re
from pathlib import Path

import pytest

from mini_serve_rs_b200 import engine as E

ROOT = Path(__file__).resolve().parents[1]


def header_functions():
    text = (ROOT / "include" / "ms_engine.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    names = re.findall(r"^\s*(?:int|int64_t)\s+(\w+)\s*\(", text, flags=re.M)
    return sorted(set(names))


def test_header_declares_the_expected_surface():
    names = header_functions()
    for must in ("ms_engine_create", "ms_step", "ms_seq_admit", "ms_seq_append_block", "ms_seq_release",
                 "ms_launch_paged_attention", "launch_paged_gqa_decode_tiled_f16", "launch_rmsnorm_f32"):
        assert must in names


def test_library_exports_every_declared_symbol():
    lib = E.lib()
    missing = [n for n in header_functions() if not hasattr(lib, n)]
    assert not missing, missing
    # the Python binding types every declared function
    assert set(header_functions()) <= set(E.exported_symbols())


def test_prototype_launchers_fail_closed_on_bad_arguments():
    lib = E.lib()
    assert lib.launch_rmsnorm_f32(None, None, None, 0, 1024, 1e-6) != 0
    assert lib.launch_rmsnorm_f16(None, None, None, 4, 0, 1e-6) != 0
    assert lib.launch_paged_gqa_decode_tiled_f32(None, None, None, None, None, None, 0, 16, 8, 8, 1.0) != 0
    assert lib.launch_paged_gqa_decode_tiled_bf16(None, None, None, None, None, None, 1, 16, 7, 8, 1.0) != 0


def test_engine_create_rejects_bad_configs_before_touching_a_device():
    from mini_serve_rs_b200.config import ModelConfig
    bad = ModelConfig(64, 32, 64, 2, 4, 2, 128, head_dim=8)  # head_dim 8 unsupported
    with pytest.raises(E.EngineError, match="head_dim"):
        E.Engine(bad, pool_blocks=16)
    bad2 = ModelConfig(1024, 256, 512, 2, 6, 4, 4096, head_dim=128)  # 6 % 4 != 0
    with pytest.raises(E.EngineError, match="multiple"):
        E.Engine(bad2, pool_blocks=16)


def test_error_mapping_matches_engine_error_variants():
    assert isinstance(E.error_for(E.MS_E_PRESSURE, "x"), E.CachePressure)
    assert isinstance(E.error_for(E.MS_E_QUARANTINED, "x"), E.NoHealthyWorkers)
    assert isinstance(E.error_for(E.MS_E_TOKEN_LIMIT, "x"), E.TokenLimitExceeded)
    for c in (E.MS_E_INVALID, E.MS_E_DEVICE, E.MS_E_INJECTED, E.MS_E_NOT_FOUND):
        assert isinstance(E.error_for(c, "x"), E.BackendError)
