"""The reference-side adapter (include/mlvc_b200_adapter.hpp) on the CPU:
it compiles against the reference's own headers, and the reference's backend
registry routes the name "b200" to it (without a GPU, creation then fails
inside the product library with its own error)."""

import os
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
REF = os.environ.get("MLVC_REFERENCE_DIR")


@pytest.mark.skipif(not REF or not Path(REF, "runtime", "include", "mlvc", "runtime", "backend.hpp").exists(),
                    reason="MLVC_REFERENCE_DIR does not name a reference source tree")
def test_adapter_compiles_against_reference_headers(tmp_path):
    tu = tmp_path / "adapter_tu.cpp"
    tu.write_text('#include "mlvc_b200_adapter.hpp"\n'
                  'static_assert(std::is_base_of_v<mlvc::BufferedCodecBackend, mlvc::b200_backend::B200Backend>);\n'
                  'static_assert(std::is_base_of_v<mlvc::InferenceBackend, mlvc::b200_backend::B200Backend>);\n'
                  'void register_it() { mlvc::b200_backend::register_b200_backend(false); }\n')
    out = subprocess.run(["g++", "-std=c++20", "-fsyntax-only", "-Wall", "-Werror", f"-I{REF}/core/include",
                          f"-I{REF}/runtime/include", f"-I{ROOT / 'include'}", str(tu)], capture_output=True, text=True)
    assert out.returncode == 0, out.stderr


def test_registry_routes_b200_to_the_adapter(tmp_path):
    from adapter_probe import PROBE, AdapterProbe
    if not PROBE.exists():
        pytest.skip("adapter probe not built (make -C oracle adapter REF=<reference tree>)")
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present: covered by tests/test_gpu_adapter.py")
    except ImportError:
        pass
    with pytest.raises(RuntimeError, match="mlvc-b200|CUDA|cuda|libcuda|device"):
        AdapterProbe(tmp_path, 0)
