"""flux_b200: B200 (sm_100a) implementation of Flux's SmolLM2-135M decode loop.

Importing the package registers the ``torch.ops.flux.*`` operator schemas.
Compute lives in ``libfluxb200.so`` (``python -m flux_b200.build``); without it
every operator and runtime raises instead of falling back to the CPU.

Public surface (the reference's names):

* ``flux_b200.integration.enable_flux_ops`` -- operator categories on a
  Hugging Face ``LlamaForCausalLM`` (``flux/model/smollm2_flux.py``);
* ``flux_b200.runtime.NativeSmolLM2Decode`` / ``NativeSmolLM2Prefill`` /
  ``native_smollm2_greedy_generate`` (``flux/runtime/native_smollm2.py``);
* ``flux_b200.operators`` -- ``*_native`` entry points (``flux/ops``).
"""

from flux_b200 import operators  # noqa: F401  (registers torch.ops.flux.*)
from flux_b200._native import LIBRARY_PATH, NativeLibraryUnavailable, is_available

__all__ = ["LIBRARY_PATH", "NativeLibraryUnavailable", "is_available", "operators"]
