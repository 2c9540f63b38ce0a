"""Run router-ia's own pytest suite with this package's
``router_ia.qwen36_attention_cache`` in place of the reference module.

``router-ia_b200`` goes first on PYTHONPATH and the reference's ``v2/src``
second; ``router_ia/__init__.py`` extends the package path, so the
reference's other modules (``qwen36_chat_batch`` ...) import our cache module
through ``from . import qwen36_attention_cache``.  Needs a router-ia checkout
(``ROUTER_IA_REFERENCE``, default /root/reference); skipped without one.
"""

from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
REF = Path(os.environ.get("ROUTER_IA_REFERENCE", "/root/reference"))


@pytest.mark.skipif(not (REF / "v2" / "tests").is_dir(), reason="no router-ia checkout")
def test_reference_v2_suite_passes_against_this_module(tmp_path):
    probe = (
        "import router_ia.qwen36_attention_cache as m, router_ia.qwen36_chat_batch as c;"
        "print(m.__file__); print(c.attention_cache.__file__)"
    )
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "router-ia_b200"), str(REF / "v2" / "src")])
    out = subprocess.run([sys.executable, "-c", probe], env=env, capture_output=True, text=True, cwd=tmp_path)
    assert out.returncode == 0, out.stderr
    ours = str((REPO / "router-ia_b200" / "router_ia" / "qwen36_attention_cache.py").resolve())
    assert out.stdout.split() == [ours, ours]
    res = subprocess.run(
        [sys.executable, "-m", "pytest", "-q", "-p", "no:cacheprovider", str(REF / "v2" / "tests")],
        env=env, capture_output=True, text=True, cwd=tmp_path, timeout=600,
    )
    assert res.returncode == 0, res.stdout[-4000:] + res.stderr[-2000:]
    assert " passed" in res.stdout
