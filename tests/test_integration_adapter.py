"""The adapter INTEGRATION.md gives a maintainer (B200RecModels, the library behind
carbon::PipelineModels) compiles against the reference's own interface headers and this
library's C header, and overrides every pure virtual (a concrete class).  Runs where the
reference tree is present (this check reads its headers; it is skipped elsewhere)."""
import re
import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
from oracle import oracle as O  # noqa: E402

REF_INCLUDE = O.REFERENCE_ROOT / "carbon" / "include"


@pytest.mark.skipif(not (REF_INCLUDE / "carbon" / "pipeline.h").exists() or shutil.which("g++") is None,
                    reason="the reference's headers or g++ are not on this machine")
def test_adapter_compiles_against_reference_pipeline_models(tmp_path):
    md = (ROOT / "INTEGRATION.md").read_text()
    code = re.search(r"```cpp\n(.*?)```", md, re.S).group(1)
    src = tmp_path / "adapter.cpp"
    src.write_text(code + "\n#include <type_traits>\n"
                   "static_assert(!std::is_abstract_v<carbon::B200RecModels>, \"every pure virtual overridden\");\n")
    r = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", f"-I{REF_INCLUDE}", f"-I{ROOT / 'include'}", str(src)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
