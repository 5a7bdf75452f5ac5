"""The reference's native ABI on librl2, without a GPU: every ``rl_*`` entry point that the
reference's ctypes code declares is exported, ``include/rl_compat.h`` declares it with the
same argument and result kinds, and argument errors are reported the reference's way
(-1 / NULL / SIZE_MAX and a message in ``rl_last_error``) before any device work."""

import ctypes
import json
import re
import subprocess
import sys
from pathlib import Path

import pytest

from oracle import build_ref
from tests._rl_abi import TABLE, bound_library, ints, pointers, sizes

ROOT = Path(__file__).resolve().parents[1]


def _header_prototypes() -> dict[str, tuple[str, list[str]]]:
    text = (ROOT / "include" / "rl_compat.h").read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    text = "\n".join(ln for ln in text.splitlines() if not ln.lstrip().startswith(("#", "extern", "}")))
    out = {}
    for ret, name, args in re.findall(r"([A-Za-z_][\w\s\*]*?)\s*\b(rl_\w+)\s*\(([^)]*)\)\s*;", text):
        ret = " ".join(ret.replace("*", " * ").split()).replace(" *", "*")
        params = [] if args.strip() in ("", "void") else [" ".join(a.replace("*", " * ").split()) for a in args.split(",")]
        out[name] = (ret, params)
    return out


def _param_kind(decl: str) -> str:
    toks = decl.split()
    stars = toks.count("*")
    base = [t for t in toks[:-1] if t not in ("const", "*")]  # drop the parameter name
    if stars >= 2:
        return "ptr*"
    if stars == 1:
        return {"size_t": "size*", "int": "int*"}.get(base[0], "ptr")
    return {"int": "int", "size_t": "size", "float": "float", "double": "double"}[base[0]]


def _return_kind(ret: str) -> str:
    return {"const char*": "str", "void*": "ptr", "int": "int", "size_t": "size"}[ret]


def test_every_reference_entry_point_is_exported():
    lib = bound_library()  # raises AttributeError on a missing export
    assert len(TABLE) == 36
    for name in TABLE:
        assert getattr(lib, name).argtypes is not None


def test_header_matches_reference_declarations():
    protos = _header_prototypes()
    assert set(protos) == set(TABLE)
    for name, sig in TABLE.items():
        ret, params = protos[name]
        assert _return_kind(ret) == sig["restype"], name
        assert [_param_kind(p) for p in params] == sig["argtypes"], name


def _err(lib) -> str:
    return lib.rl_last_error().decode()


def test_argument_errors_follow_reference_convention():
    lib = bound_library()
    assert lib.rl_plan_create(0, 4, 4, 0, 0, 4, 4, 4, 0, 0, 0) is None
    assert _err(lib) == "Dense dimensions must be positive."
    assert lib.rl_plan_create(4, 4, 4, 2, 0, 4, 4, 4, 0, 0, 0) is None
    assert "Transpose flags" in _err(lib)
    assert lib.rl_plan_create(8, 4, 4, 0, 0, 4, 4, 8, 0, 0, 0) is None  # lda < m
    assert "leading dimension" in _err(lib)
    assert lib.rl_plan_create_mixed(4, 4, 4, 0, 0, 4, 4, 4, 0, 1, 1, 0) is None
    assert _err(lib) == "TF32 applies only to FP32 inputs."
    assert lib.rl_plan_create(4, 4, 3_000_000, 0, 0, 4, 3_000_000, 4, 0, 0, 0) is None  # staging grid limit
    assert "K above" in _err(lib)
    assert lib.rl_plan_workspace(None) == ctypes.c_size_t(-1).value
    assert lib.rl_plan_tuning_metadata(None) is None
    assert lib.rl_plan_run(None, None, None, None, None, None, None, 0, 0.0, None) == -1
    assert lib.rl_plan_destroy(None) == 0
    assert lib.rl_cast_f32_f16(None, None, 0, None) == -1
    assert lib.rl_bias_grad(None, None, 0, 4, None) == -1

    fake = pointers([0x1000])
    assert lib.rl_adam_create(1, fake, fake, fake, fake, sizes([4]), 0x1000, 0x1000, 1.0, 0.999, 1e-8) is None
    assert "betas" in _err(lib)
    assert lib.rl_adam_create(0, fake, fake, fake, fake, sizes([4]), 0x1000, 0x1000, 0.9, 0.999, 1e-8) is None
    assert lib.rl_adam_unscale(None, None) == -1
    assert lib.rl_adam_step(None, None) == -1
    assert lib.rl_adam_set_scaler(None, *([None] * 6), 2.0, 0.5, 2000) == -1

    assert lib.rl_flash_projection_create(1, fake, fake, sizes([4]), ints([3])) is None
    assert _err(lib) == "Invalid projection row/vector."
    assert lib.rl_flash_projection_create_with_shadows(1, fake, fake, sizes([4]), ints([2]), fake) is None
    assert "shadows" in _err(lib)
    assert lib.rl_flash_ema_create(1, fake, fake, sizes([4]), 2.0) is None
    assert _err(lib) == "Invalid EMA metadata/tau."
    assert lib.rl_flash_projection_step(None, None) == -1
    assert lib.rl_flash_ema_step(None, None) == -1

    assert lib.rl_flash_bn_forward(*([None] * 9), 0, 4, 1e-5, 0.01, 1, 0, None) == -1
    assert "normalization" in _err(lib)
    assert lib.rl_flash_bn_forward(*([None] * 9), 4, 4, 1e-5, 0.01, 1, 0, None) == -1
    assert _err(lib) == "Invalid BN forward arrays/count."
    assert lib.rl_flash_bn_forward_with_fp16(*([None] * 10), 4, 4, 1e-5, 0.01, 1, 0, None) == -1
    assert lib.rl_flash_bn_backward(*([None] * 11), 4, 4, 0.0, 1, 0, None) == -1
    assert lib.rl_flash_bn_backward_controlled(*([None] * 12), 2, 4, 4, 1e-5, 1, 0, None) == -1
    assert lib.rl_flash_rms_forward(None, None, None, None, 4, 4, 1e-6, None) == -1
    assert lib.rl_flash_rms_backward(*([None] * 7), 4, 4, 1e-6, None) == -1

    assert lib.rl_flash_categorical_forward(*([None] * 5), 4, 1, None) == -1
    assert lib.rl_flash_categorical_backward(*([None] * 7), 4, 11, None) == -1
    assert lib.rl_flash_categorical_target(*([0x1000] * 9), 4, 4097, -10.0, 10.0, None) == -1
    assert "2..4096 bins" in _err(lib)
    assert lib.rl_flash_categorical_target(*([0x1000] * 9), 4, 11, 1.0, 1.0, None) == -1

    assert lib.rl_zero_create(2, pointers([0x2000, 0x1000]), sizes([4, 4])) is None
    assert _err(lib) == "Zero spans must be sorted and nonoverlapping."
    assert lib.rl_zero_create(2, pointers([0x1000, 0x1008]), sizes([4, 4])) is None  # overlap
    assert lib.rl_zero_create(1, pointers([0x1002]), sizes([4])) is None  # misaligned
    assert lib.rl_zero_step(None, None) == -1
    for destroy in ("rl_adam_destroy", "rl_flash_projection_destroy", "rl_flash_ema_destroy", "rl_zero_destroy"):
        assert getattr(lib, destroy)(None) == 0


def test_fixture_is_what_the_reference_declares():
    """Re-records the ctypes declarations from the reference's own code (where its sources
    are present) and compares them with the committed fixture."""
    src = build_ref.reference_root() / "src"
    if not (src / "robolearn" / "cuda" / "_runtime.py").is_file():
        pytest.skip("reference sources absent")
    code = ("import json, sys; from pathlib import Path; sys.path.insert(0, 'tests/golden'); "
            "import make_rl_abi as m; print(json.dumps(m.record(Path(sys.argv[1]))))")
    done = subprocess.run([sys.executable, "-c", code, str(src)], cwd=ROOT, capture_output=True, text=True,
                          timeout=120)
    assert done.returncode == 0, done.stderr
    assert json.loads(done.stdout.strip().splitlines()[-1]) == TABLE


def test_reference_library_build_skips_without_sources(tmp_path, monkeypatch):
    monkeypatch.setenv("RL2_REFERENCE_ROOT", str(tmp_path))
    assert build_ref.build() is None
