"""The command-line tools that mirror the reference's binaries: `attn_sm100 [B H S D]`
(src/attn_sm75.cu:442-554) and `gdn_sm100 [T]` (src/gdn_sm75.cu:1246-1412), with the
reference's exit codes (0 pass, 1 a check failed, 2 usage).

Usage errors are rejected before any CUDA call, so those run on CPU; the checks that
launch kernels are GPU tests."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "turing-sm75_b200", "bin")


def _run(name, *args, timeout=300):
    exe = os.path.join(BIN, name)
    if not os.path.exists(exe):
        pytest.skip(f"{name} not built")
    return subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("args", [("2", "8", "512", "96"),      # head dim not built
                                  ("2", "8", "512"),            # three positionals
                                  ("2", "8", "2048", "128"),    # naive check needs S <= 1024
                                  ("2", "6", "128", "128", "--hkv", "4"),  # H % Hkv != 0
                                  ("--bogus",)])
def test_attn_cli_usage_errors(args):
    r = _run("attn_sm100", *args)
    assert r.returncode == 2, (r.stdout, r.stderr)


@pytest.mark.parametrize("args", [("0",), ("4096",), ("--what",)])
def test_gdn_cli_usage_errors(args):
    r = _run("gdn_sm100", *args)
    assert r.returncode == 2, (r.stdout, r.stderr)


@pytest.mark.gpu
@pytest.mark.parametrize("args", [(), ("1", "4", "256", "128"), ("2", "8", "512", "64", "--bf16"),
                                  ("1", "6", "256", "256", "--hkv", "1", "--bf16"),
                                  ("2", "8", "300", "128", "--hkv", "2", "--causal", "0")])
def test_attn_cli_passes(cuda, args):
    r = _run("attn_sm100", *args, "--iters", "2")
    assert r.returncode == 0, (r.stdout, r.stderr)
    assert "max |tcgen05-naive|" in r.stdout and " OK" in r.stdout, r.stdout


@pytest.mark.gpu
@pytest.mark.parametrize("T", ["64", "200"])
def test_gdn_cli_passes(cuda, T):
    r = _run("gdn_sm100", T, "--iters", "1")
    assert r.returncode == 0, (r.stdout, r.stderr)
    assert "FAIL" not in r.stdout and "OK" in r.stdout, r.stdout
