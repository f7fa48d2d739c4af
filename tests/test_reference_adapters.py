"""The reference's own consumers, unmodified, on this package.

The reference ships a vLLM block manager and an SGLang radix cache
(integrations/vllm/block_manager.py, integrations/sglang/radix_cache.py)
with tests that run them over stand-ins of vLLM and SGLang
(tests/test_vllm_integration.py, tests/test_sglang_integration.py,
tests/fakes/).  Here those test files run, as they are, in a child pytest
with agentkv_b200 registered under the reference's module names
(tests/reference_alias_plugin.py): every CoW pair, block table, hit length
and eviction count the tests check comes from this package's AgentKVPool
and DualRadixTree.  With no GPU the allocator and the tree kernels are the
suite's CPU stand-ins (the oracle's allocator, the tree kernels' CPU model).

Needs a checkout of the reference, named by the AGENTKV_REFERENCE
environment variable; skipped without one.  Nothing is written into the
checkout (no byte code, no pytest cache).
"""

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parent.parent
REF = os.environ.get("AGENTKV_REFERENCE")

pytestmark = pytest.mark.skipif(
    not REF or not (Path(REF) / "integrations").is_dir() or not (Path(REF) / "tests" / "fakes").is_dir(),
    reason="set AGENTKV_REFERENCE to a checkout of the reference to run its adapter tests here")


@pytest.mark.parametrize("name", ["test_vllm_integration.py", "test_sglang_integration.py"])
def test_reference_adapter_tests_pass_on_this_package(name, tmp_path):
    env = dict(os.environ, PYTHONDONTWRITEBYTECODE="1",
               PYTHONPATH=os.pathsep.join([str(REPO / "tests"), str(REPO), REF]))
    cmd = [sys.executable, "-m", "pytest", str(Path(REF) / "tests" / name), "-p", "reference_alias_plugin",
           "-p", "no:cacheprovider", "-q", "-s", "-x", "--rootdir", str(tmp_path), "-c", os.devnull,
           "-W", "ignore::DeprecationWarning"]
    proc = subprocess.run(cmd, cwd=tmp_path, env=env, capture_output=True, text=True, timeout=600)
    out = proc.stdout + proc.stderr
    assert proc.returncode == 0, out[-4000:]
    assert " passed" in out and " failed" not in out, out[-2000:]
    # the adapters ran on this package, not on the reference's own
    line = next(x for x in out.splitlines() if x.startswith("agentkv_b200 alias:"))
    fields = dict(f.split("=") for f in line.split(": ", 1)[1].split())
    assert fields["aliased"] == "True", line
    assert int(fields["pools"]) >= 5 and int(fields["lookups"]) >= 5, line
