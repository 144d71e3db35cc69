"""Numbers in parameters, model JSON and the configuration are read and
written with '.' as the decimal point whatever locale the host process has
set, as XGBoost's own parsers do.  A process that calls setlocale with a
decimal-comma LC_NUMERIC (a GUI or a localised CLI) must still load models
and accept "0.3".  The test builds such a locale with localedef into a
temporary directory and runs the checks in a child process, so the locale
change stays out of the test runner."""
import pathlib
import shutil
import subprocess
import sys
import textwrap

import pytest

ROOT = pathlib.Path(__file__).resolve().parents[1]

LOCALE_SRC = """comment_char %
escape_char /
LC_NUMERIC
decimal_point "<U002C>"
thousands_sep ""
grouping -1
END LC_NUMERIC
"""
CHARMAP = """<code_set_name> ASCIIMIN
<comment_char> %
<escape_char> /
CHARMAP
<U002C> /x2c COMMA
<U002E> /x2e FULL STOP
END CHARMAP
"""

CHILD = textwrap.dedent("""
    import ctypes, json, sys
    sys.path[:0] = [sys.argv[1] + "/decision-programs_b200", sys.argv[1] + "/tests"]
    libc = ctypes.CDLL(None)
    libc.setlocale.restype = ctypes.c_char_p
    libc.setlocale.argtypes = [ctypes.c_int, ctypes.c_char_p]
    assert libc.setlocale(1, b"comma_test") == b"comma_test"      # LC_NUMERIC
    libc.strtod.restype = ctypes.c_double
    libc.strtod.argtypes = [ctypes.c_char_p, ctypes.c_void_p]
    assert libc.strtod(b"0,5", None) == 0.5                        # the locale is in force
    import dp_gbdt as dp
    from test_abi import _model
    L, C = dp.lib(), ctypes
    h = C.c_void_p()
    assert L.XGBoosterCreate(None, 0, C.byref(h)) == 0
    for k, v in ((b"eta", b"0.3"), (b"lambda", b"1.5"), (b"subsample", b"0.75"), (b"base_score", b"[0.25]")):
        assert L.XGBoosterSetParam(h, k, v) == 0, (k, L.XGBGetLastError())
    m = _model()
    m["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"] = [0.1, -1.25, 0.3]
    buf = json.dumps(m).encode()
    assert L.XGBoosterLoadModelFromBuffer(h, buf, len(buf)) == 0, L.XGBGetLastError()
    n, p = C.c_uint64(), C.c_void_p()
    assert L.XGBoosterSaveModelToBuffer(h, b'{"format":"json"}', C.byref(n), C.byref(p)) == 0
    saved = json.loads(C.string_at(p, n.value))
    conds = saved["learner"]["gradient_booster"]["model"]["trees"][0]["split_conditions"]
    assert conds == [0.1, -1.25, 0.3], conds
    s = C.c_char_p()
    assert L.XGBoosterSaveJsonConfig(h, C.byref(n), C.byref(s)) == 0
    cfg = json.loads(C.string_at(s, n.value))
    print("ok", cfg["learner"]["gradient_booster"]["tree_train_param"]["eta"]
          if "tree_train_param" in cfg["learner"]["gradient_booster"] else "")
""")


def test_numbers_ignore_a_decimal_comma_locale(dp, tmp_path):
    localedef = shutil.which("localedef")
    if localedef is None:
        pytest.skip("localedef is not installed")
    (tmp_path / "src").write_text(LOCALE_SRC)
    (tmp_path / "charmap").write_text(CHARMAP)
    subprocess.run([localedef, "-c", "-i", str(tmp_path / "src"), "-f", str(tmp_path / "charmap"),
                    str(tmp_path / "comma_test")], capture_output=True, timeout=120)
    if not (tmp_path / "comma_test" / "LC_NUMERIC").exists():
        pytest.skip("localedef could not build the test locale")
    r = subprocess.run([sys.executable, "-c", CHILD, str(ROOT)], capture_output=True, text=True, timeout=300,
                       env={"LOCPATH": str(tmp_path), "PATH": "/usr/bin:/bin"})
    assert r.returncode == 0 and r.stdout.startswith("ok"), r.stdout + r.stderr
