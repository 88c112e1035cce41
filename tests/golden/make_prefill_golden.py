"""Golden vectors for the benchmark's 8192-token prefill.

Runs the reference's FP32 path -- transformers ``LlamaForCausalLM`` eager on
the CPU, as ``benchmarks/benchmark_flux.py:533-564`` drives it -- on the
benchmark's own inputs (SmolLM2-135M geometry, seed-0 weights, the seed-0
uniform 8192-token prompt) and stores what a GPU test can compare cheaply:

* ``logits``: the last prompt position's logits ``[49152]``;
* ``key_sums`` / ``value_sums``: per layer and KV head, the FP64 sum and sum
  of squares of the cached (post-RoPE) keys and the values over all 8192 rows
  ``[30, 3, 2]``;
* ``rows`` / ``key_rows`` / ``value_rows``: full cache rows at a few
  positions ``[30, 3, len(rows), 64]``.

    python tests/golden/make_prefill_golden.py      # ~5 min on 8 cores, ~20 GB RAM
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parents[1]))

from tests.golden.inputs import build_model, smollm2_config, uniform_prompt  # noqa: E402
from tests.host import limit_threads  # noqa: E402

CONTEXT = 8192
ROWS = (0, 1, 127, 4095, 8190, 8191)


def main() -> None:
    limit_threads()
    model = build_model(smollm2_config(), 0)
    prompt = uniform_prompt(CONTEXT, seed=0)
    with torch.inference_mode():
        out = model(input_ids=prompt, use_cache=True, logits_to_keep=1)
    layers = out.past_key_values.layers
    keys = [layer.keys[0].double() for layer in layers]      # [3, 8192, 64] per layer
    values = [layer.values[0].double() for layer in layers]

    def sums(tensors):
        return np.stack([torch.stack([t.sum(dim=(1, 2)), (t * t).sum(dim=(1, 2))], dim=-1).numpy() for t in tensors])

    np.savez_compressed(
        HERE / "prefill8192.npz",
        logits=out.logits[0, -1].float().numpy(),
        key_sums=sums(keys), value_sums=sums(values), rows=np.array(ROWS, np.int64),
        key_rows=np.stack([k[:, list(ROWS)].float().numpy() for k in keys]),
        value_rows=np.stack([v[:, list(ROWS)].float().numpy() for v in values]))
    print("wrote", HERE / "prefill8192.npz")


if __name__ == "__main__":
    main()
