from __future__ import annotations

import importlib
import json
import os
import sys
from pathlib import Path

import numpy as np
import pytest

REPO_ROOT = Path(__file__).resolve().parents[1]
if str(REPO_ROOT) not in sys.path:
    sys.path.insert(0, str(REPO_ROOT))

GOLDEN_DIR = Path(__file__).resolve().parent / "golden"

# the reference package (extended_einsum, pure Python), installed unmodified by
# baseline/install_reference.sh; XE_REFERENCE_PACKAGE points elsewhere
REFERENCE_PACKAGE = Path(os.environ.get("XE_REFERENCE_PACKAGE", REPO_ROOT / "baseline" / "_ref"))

# fp32 log-domain tolerance: 1e-5 absolute, plus two fp32 ulps of the
# reference value (below 1e-5 for |value| < 40; the fp32 representation of
# larger log-values cannot resolve 1e-5, e.g. ulp(1000) = 6.1e-5).
LOG_ATOL = 1e-5
LOG_RTOL = 2.4e-7


def pytest_configure(config: pytest.Config) -> None:
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def pytest_collection_modifyitems(config: pytest.Config, items: list[pytest.Item]) -> None:
    # keep GPU tests ordered after CPU tests inside a module-agnostic run
    items.sort(key=lambda item: ("gpu" in item.keywords, item.fspath.basename.startswith("test_zz")))


def import_reference():
    """Imports the reference package from REFERENCE_PACKAGE; skips the test when it is not installed."""
    if not (REFERENCE_PACKAGE / "extended_einsum").is_dir():
        pytest.skip(f"reference package not installed in {REFERENCE_PACKAGE} (baseline/install_reference.sh)")
    if str(REFERENCE_PACKAGE) not in sys.path:
        sys.path.insert(0, str(REFERENCE_PACKAGE))
    return importlib.import_module("extended_einsum")


@pytest.fixture(scope="session")
def reference_xe():
    return import_reference()


@pytest.fixture(scope="session")
def golden() -> dict[str, np.ndarray]:
    with np.load(GOLDEN_DIR / "golden.npz") as data:
        return {k: data[k] for k in data.files}


@pytest.fixture(scope="session")
def golden_programs() -> dict[str, dict]:
    return json.loads((GOLDEN_DIR / "programs.json").read_text())


def build_program(spec: dict, mode: str):
    """Rebuilds a serialized golden program with extended_einsum_b200's IR classes."""
    from extended_einsum_b200 import frontend as fe

    classes = {
        "exp": lambda a: fe.OperatorExp(),
        "log": lambda a: fe.OperatorLog(),
        "+": lambda a: fe.OperatorAdd(),
        "-": lambda a: fe.OperatorSubtract(),
        "*": lambda a: fe.OperatorMultiply(),
        "/": lambda a: fe.OperatorDivide(),
        "stack": lambda a: fe.OperatorStack(a["axis"]),
        "concat": lambda a: fe.OperatorConcat(a["axis"]),
        "take": lambda a: fe.OperatorTake(a["axis"]),
        "select": lambda a: fe.OperatorSelect(a["axis"], a["index"]),
        "slice": lambda a: fe.OperatorSlice(a["start"], a["stop"], a["axis"]),
        "softmax": lambda a: fe.OperatorSoftmax(tuple(a["axis"]) if isinstance(a["axis"], list) else a["axis"]),
        "einsum": lambda a: fe.OperatorEinsum(a["format_string"]),
    }
    instructions = [fe.RichInstruction(classes[name](attrs), tuple(args)) for name, attrs, args in spec["instructions"]]
    return fe.RichProgram(
        instructions=instructions,
        n_inputs=spec["n_inputs"],
        stability_mode=mode,
        tensor_formats=["dense"] * (spec["n_inputs"] + len(instructions)),
        shapes=[tuple(s) for s in spec["shapes"]],
        parameter_indices=frozenset(spec["parameter_indices"]),
    )


def golden_inputs(golden: dict, name: str, spec: dict) -> list[np.ndarray]:
    return [golden[f"{name}/in{i}"] for i in range(spec["n_inputs"])]


def log_close(actual: np.ndarray, expected: np.ndarray, atol: float = LOG_ATOL, rtol: float = LOG_RTOL) -> None:
    """Elementwise |actual - expected| <= atol + rtol*|expected|, with matching non-finite values."""
    actual = np.asarray(actual, dtype=np.float64)
    expected = np.asarray(expected, dtype=np.float64)
    assert actual.shape == expected.shape, (actual.shape, expected.shape)
    np.testing.assert_allclose(actual, expected, atol=atol, rtol=rtol, equal_nan=True)
