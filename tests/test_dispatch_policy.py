"""MINICPM_W8A8_DECODE policy (src/csrc/lib/language_model.cpp:19-41 and
decoder_layer.cpp:19-25), host side only: the mode table, the environment
read once per process, and the programmatic override."""
import os
import subprocess
import sys

import pytest

import mcv_b200
from conftest import ROOT

TOKENS = ["mlp", "linear_qkv", "linear_z", "linear_out", "full_q", "full_k", "full_v", "full_o", "lm_head"]


def expected(mode, token):
    """The reference's rule, restated."""
    if mode in ("", "0", "false"):
        return False
    if mode == "all":
        return True
    if mode in ("1", "selective"):
        return token == "lm_head"
    return token in mode


@pytest.mark.parametrize("mode", ["", "0", "false", "all", "1", "selective", "mlp", "mlp,lm_head",
                                  "full", "linear_qkv+full_o", "true"])
def test_policy_table(mode):
    for t in TOKENS:
        assert mcv_b200.w8a8_policy_allows(t, mode=mode) == expected(mode, t), (mode, t)


def _in_fresh_process(env_mode, code):
    env = dict(os.environ)
    if env_mode is None:
        env.pop("MINICPM_W8A8_DECODE", None)
    else:
        env["MINICPM_W8A8_DECODE"] = env_mode
    pkg = os.path.join(ROOT, "minicpm-v-4.6-orangepi_b200")
    out = subprocess.run([sys.executable, "-c", f"import sys; sys.path.insert(0, {pkg!r}); import mcv_b200 as m; {code}"],
                         env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    return out.stdout.strip()


def expected_gate(env_mode):
    """decoder_layer.cpp:19-25: set (even empty) and neither "0" nor "false"."""
    return env_mode is not None and env_mode not in ("0", "false")


@pytest.mark.parametrize("env_mode", [None, "", "0", "false", "all", "selective", "mlp,full_q"])
def test_policy_from_environment(env_mode):
    code = ("print(int(m.w8a8_decode_enabled()), int(m.w8a8_decode_gate_enabled()), "
            "''.join(str(int(m.w8a8_policy_allows(t))) for t in %r))" % TOKENS)
    got = _in_fresh_process(env_mode, code)
    mode = env_mode or ""
    want = (f"{int(mode not in ('', '0', 'false'))} {int(expected_gate(env_mode))} "
            + "".join(str(int(expected(mode, t))) for t in TOKENS))
    assert got == want


def test_override_then_back_to_environment():
    code = ("m.set_w8a8_decode_mode('all'); a = m.w8a8_policy_allows('mlp'); "
            "m.set_w8a8_decode_mode('0'); b = m.w8a8_decode_enabled(); "
            "m.set_w8a8_decode_mode(None); c = m.w8a8_policy_allows('lm_head'), m.w8a8_policy_allows('mlp'); "
            "print(int(a), int(b), int(c[0]), int(c[1]))")
    assert _in_fresh_process("selective", code) == "1 0 1 0"
