"""Small fixed workloads for ncu captures (the commands in ``profiles/``).

    python -m tests.profile_workloads {tc-gemm,prefill,batched} [--context N] [--batch B] [--seed S]

* ``tc-gemm``: three 8192 x 576 -> 3072 3xTF32 tensor-core projections
  through ``fx_linear_3xtf32_f32`` (the prefill's largest GEMM shape).
* ``prefill``: one native prefill of a seeded ``--context``-token prompt.
* ``batched``: two batched decode steps of ``--batch`` sequences with ragged
  seeded contexts in ``--contexts LOW HIGH`` (default [512, 4096], the
  benchmark's batched configuration; a multi-pass capture of the projections
  uses short contexts, since the GEMMs do not depend on them and the caches
  then stay small).

Each prints ``<name> ok`` and exits 0; nothing is timed here (a number printed
by a run under a profiler is not a measurement).
"""

from __future__ import annotations

import argparse
import copy
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

BATCH_CONTEXT = (512, 4096)


def _model(context: int, seed: int, device):
    from flux_b200.integration import FINAL_FLUX_OPERATOR_CATEGORIES, enable_flux_ops
    from tests.golden.inputs import build_model, smollm2_config
    config = smollm2_config(vocab_size=49152, max_positions=max(8320, context + 8))
    return enable_flux_ops(copy.deepcopy(build_model(config, seed)).to(device),
                           operators=FINAL_FLUX_OPERATOR_CATEGORIES)


def tc_gemm(args, device) -> None:
    from flux_b200 import _native
    lib = _native.load()
    g = torch.Generator(device=device).manual_seed(args.seed)
    m, k, n = 8192, 576, 3072
    x = torch.randn(m, k, device=device, generator=g)
    w = torch.randn(n, k, device=device, generator=g) * 0.02
    hi, lo, out = torch.empty_like(w), torch.empty_like(w), torch.empty(m, n, device=device)
    err = torch.zeros(1, dtype=torch.int32, device=device)
    stream = torch.cuda.current_stream(device).cuda_stream
    _native.check(lib.fx_tf32_split_f32(w.data_ptr(), hi.data_ptr(), lo.data_ptr(), w.numel(), stream))
    for _ in range(3):
        _native.check(lib.fx_linear_3xtf32_f32(x.data_ptr(), hi.data_ptr(), lo.data_ptr(), None, out.data_ptr(),
                                               m, k, n, err.data_ptr(), stream))
    torch.cuda.synchronize()
    assert int(err.item()) == 0


def prefill(args, device) -> None:
    from flux_b200.runtime import NativeSmolLM2Prefill
    from tests.golden.inputs import uniform_prompt
    model = _model(args.context, args.seed, device)
    with torch.inference_mode():
        NativeSmolLM2Prefill.capture(model, uniform_prompt(args.context, seed=args.seed).to(device),
                                     max_decode_steps=1)
    torch.cuda.synchronize()


def batched(args, device) -> None:
    from flux_b200 import sharding
    from flux_b200.runtime import NativeSmolLM2BatchedDecode
    model = _model(BATCH_CONTEXT[1], args.seed, device)
    low, high = args.contexts
    lengths, tokens = sharding.shard_contexts(args.seed, sharding.sequence_shard(args.batch, 1, 0), low, high)
    runtime = NativeSmolLM2BatchedDecode(model, args.batch, high + 8)
    dgen = torch.Generator(device=device)
    with torch.inference_mode():
        for i, n in enumerate(lengths):
            dgen.manual_seed(args.seed * 1_000_003 + 29 + i)
            keys = torch.randn(30, 3, n, 64, device=device, generator=dgen) * 0.5
            values = torch.randn(30, 3, n, 64, device=device, generator=dgen) * 0.5
            runtime.load(i, tokens[i], list(keys), list(values), n)
        runtime.step(2)
        runtime.check()
    torch.cuda.synchronize()


WORKLOADS = {"tc-gemm": tc_gemm, "prefill": prefill, "batched": batched}


def main(argv=None) -> int:
    p = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    p.add_argument("workload", choices=sorted(WORKLOADS))
    p.add_argument("--context", type=int, default=8192)
    p.add_argument("--batch", type=int, default=64)
    p.add_argument("--seed", type=int, default=0)
    p.add_argument("--contexts", type=int, nargs=2, default=list(BATCH_CONTEXT), metavar=("LOW", "HIGH"))
    args = p.parse_args(argv)
    from tests.host import limit_threads
    limit_threads()
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    WORKLOADS[args.workload](args, device)
    print(f"{args.workload} ok", flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
