"""CPU tests of the C ABI library: it loads, exports every declared symbol, and its
host-side logic (synthetic generator, X4 packer) is deterministic and matches
the packer semantics.  No compute entry point is called without a GPU."""
import ctypes as C
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def _declared(header: Path, prefix: str) -> set[str]:
    text = header.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(rf"\b({prefix}\w+)\s*\(", text))


def test_libzgpu_exports_every_declared_symbol():
    from zero_b200 import _lib

    lib = C.CDLL(str(_lib.LIB_PATH))
    declared = _declared(ROOT / "include" / "zgpu.h", "zgpu_")
    assert len(declared) > 25
    missing = [s for s in sorted(declared) if not hasattr(lib, s)]
    assert not missing, f"declared in zgpu.h but not exported: {missing}"
    # every binding the Python layer uses is declared in the header
    assert set(_lib.EXPORTED) <= declared


def test_integration_notes_bind_every_declared_symbol():
    """INTEGRATION.md's Rust extern blocks declare every entry point of
    zgpu.h (the binding a maintainer adds to the crate)."""
    declared = _declared(ROOT / "include" / "zgpu.h", "zgpu_")
    notes = (ROOT / "INTEGRATION.md").read_text()
    bound = set(re.findall(r"pub fn (zgpu_\w+)\s*\(", notes))
    missing = sorted(declared - bound)
    assert not missing, f"no Rust binding in INTEGRATION.md for: {missing}"


def test_liboracle_exports_every_declared_symbol():
    import oracle

    declared = _declared(ROOT / "oracle" / "zoracle.h", "zo_")
    missing = [s for s in sorted(declared) if not hasattr(oracle.LIB, s)]
    assert not missing


def test_product_library_links_no_oracle():
    # The product must never route through the checker.
    import subprocess

    from zero_b200 import _lib

    syms = subprocess.run(["nm", "-D", str(_lib.LIB_PATH)], capture_output=True, text=True).stdout
    assert " zo_" not in syms
    for py in (ROOT / "zero_b200").rglob("*.py"):
        src = py.read_text()
        assert "import oracle" not in src and "from oracle" not in src, py


def test_status_strings_cover_all_codes():
    import zero_b200 as zb
    from zero_b200._lib import LIB

    for code in zb.STATUS:
        assert LIB.zgpu_status_string(code).decode() != "unknown status"


def test_init_without_device_reports_no_device():
    import zero_b200 as zb

    try:
        import torch

        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    with pytest.raises(zb.ZgpuError) as e:
        zb.Context()
    assert e.value.status == 90


def test_synth_is_deterministic_and_counter_based():
    from zero_b200 import synth

    a = synth.q4_0(7, 3, 8, 64, 0.02)
    b = synth.q4_0(7, 3, 8, 64, 0.02)
    assert np.array_equal(a, b)
    # rows are independent of how many rows were generated
    big = synth.q4_0(7, 3, 200, 64, 0.02)
    assert np.array_equal(big[: a.size], a)
    assert not np.array_equal(a, synth.q4_0(8, 3, 8, 64, 0.02))
    q8 = synth.q8_0(7, 4, 4, 64, 0.02 / 127).reshape(-1, 34)
    qs = q8[:, 2:].view(np.int8)
    assert qs.min() >= -127 and qs.max() <= 127
    assert np.all(q8[:, 0] | (q8[:, 1].astype(np.uint16) << 8) == q8[0, 0] | (q8[0, 1].astype(np.uint16) << 8))


def test_synth_q4_scale_distribution():
    from zero_b200 import synth

    w = synth.q4_0(1, 9, 512, 2048, 0.02).reshape(-1, 18)
    d = w[:, :2].copy().view(np.float16).astype(np.float64).ravel()
    # |N(0, 0.02)| / 8 has mean 0.02 * sqrt(2/pi) / 8
    assert abs(d.mean() - 0.02 * np.sqrt(2 / np.pi) / 8) < 2e-5
    nib = np.concatenate([w[:, 2:] & 0xF, w[:, 2:] >> 4]).ravel()
    assert abs(nib.mean() - 7.5) < 0.05


def test_pack_x4_rejects_partial_groups():
    from zero_b200 import synth

    with pytest.raises(ValueError):
        synth.pack_x4(np.zeros(6 * 2 * 18, np.uint8), 6, 64, "q4_0")


def test_weight_bytes_per_token_config0():
    from zero_b200 import synth

    cfg = synth.QWEN3_1_7B
    # 28 x 28,311,552 (Q4_0 matmuls) + 330,612,736 (Q8_0 LM head) + norms + one embedding row
    assert cfg.weight_bytes_per_token() == 28 * 28311552 + 330612736 + 4 * (2 * 28 * 2048 + 2 * 28 * 128 + 2048) + 2176
