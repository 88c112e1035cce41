"""One process driving two GPUs: every kernel's shared-memory limit is set
per CUDA context, so runtimes and operators on a second device run (and give
the same results as on the first) without a process of their own.  Needs two
visible GPUs; skipped otherwise."""

from __future__ import annotations

import copy

import numpy as np
import pytest
import torch

from oracle import hf_reference as hf
from tests.golden import inputs as gi

pytestmark = pytest.mark.gpu


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_runtimes_on_two_devices_in_one_process(tiny30_model):
    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    from flux_b200.runtime import NativeSmolLM2Prefill
    ids = gi.tiny30_ids(17)
    logits = []
    for device in ("cuda:0", "cuda:1"):
        torch.cuda.set_device(device)
        model = enable_flux_ops(copy.deepcopy(tiny30_model).to(device), operators=FINAL_FLUX_OPERATOR_CATEGORIES)
        with torch.inference_mode():
            native = NativeSmolLM2Prefill.capture(model, ids.to(device), max_decode_steps=3)
            steps = [native.logits.reshape(-1).cpu().numpy()]
            token = torch.argmax(native.logits, dim=-1).view(1, 1)
            for _ in range(3):
                out = native.replay(token)
                steps.append(out.reshape(-1).cpu().numpy())
                token = torch.argmax(out, dim=-1).view(1, 1)
        logits.append(np.stack(steps))
        del native, model
    torch.cuda.set_device("cuda:0")
    # deterministic kernels: the two devices agree bit for bit
    np.testing.assert_array_equal(logits[0], logits[1])


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_attention_op_on_two_devices_in_one_process():
    from flux_b200 import operators as ops
    q, k, v, m = gi.gqa_inputs(1024)
    outs = []
    for device in ("cuda:1", "cuda:0"):  # the second device first
        with torch.cuda.device(device):
            out = ops.gqa_decode_attention_native(q.to(device), k.to(device), v.to(device), None, 0.125,
                                                  torch.tensor(777, device=device))
            outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1])
    assert hf is not None
