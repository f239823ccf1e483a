"""Host-side pieces of bench.py: the roofline's byte count, the traffic lookup in the committed
ncu summaries, and the config both arms print. No GPU."""
import importlib.util
import re
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_under_test", ROOT / "bench.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_compulsory_bytes_by_hand(bench):
    from appt_spgemm.matrices import Csr
    # rows 1..2 of A touch B rows {0, 2} and {2}: B rows 0 (2 entries) and 2 (1 entry)
    A = Csr(3, 3, np.array([0, 1, 3, 4], np.int32), np.array([1, 0, 2, 2], np.int32),
            np.ones(4))
    B_rp = np.array([0, 2, 3, 4], np.int32)
    got = bench.compulsory_bytes(A, B_rp, 1, 3, c_nnz=5)
    m, a_nnz = 2, 3
    want = (4 * (m + 1) + 12 * a_nnz) + (12 * (2 + 1) + 8 * 2) + (8 * (m + 1) + 12 * 5)
    assert got == want


def test_traffic_lookup_matches_workload_and_rows(bench):
    t, src = bench.traffic_from_profiles("numeric_stencil27", "stencil27_64cube_AxA", 262144)
    assert t == 1009074944 and src == "profiles/numeric_stencil27.txt"
    # a summary is used only for the workload and row count it names
    assert bench.traffic_from_profiles("numeric_stencil27", "stencil27_64cube_AxA", 34480) == \
        (None, None)
    assert bench.traffic_from_profiles("numeric_nothing", "x", 1) == (None, None)


def test_scaled_traffic_follows_its_stated_factor(bench):
    """The banded summary is a 2^20-row capture scaled to the 2^22-row launch by the rows of the
    launch; the scaled figure must be the captured one times that ratio."""
    t, src = bench.traffic_from_profiles("numeric_banded", "banded_2^22_w256_AxA", 4194304)
    assert src == "profiles/numeric_banded_2e20.txt"
    text = (ROOT / src).read_text()
    captured = int(re.search(r"traffic bytes \(read \+ write\)\s+(\d+)", text).group(1))
    ratio = 4039797 / 1009630
    assert abs(t - captured * ratio) <= 1


def test_every_profile_names_its_command():
    for f in sorted((ROOT / "profiles").glob("*.txt")):
        text = f.read_text()
        assert "ncu " in text and "--clock-control none" in text, f.name
        if "traffic_bytes_per_launch:" in text:
            assert re.search(r"^workload: \S+ rows=\d+$", text, re.M), f.name


def test_config_keys(bench):
    from appt_spgemm.matrices import Csr
    A = Csr(2, 2, np.array([0, 1, 2], np.int32), np.array([0, 1], np.int32), np.ones(2))
    wl = bench._wl()["stencil27"]
    cfg = bench.config_of(wl, A, 2, 2, "adaptive", 1)
    assert set(cfg) == {"workload", "rows", "cols", "nnz_a", "nnz_c", "products", "method",
                        "parallelism"}
    assert cfg["workload"] == "stencil27_64cube_AxA"
