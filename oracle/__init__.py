"""CPU oracle for the Flux SmolLM2-135M FP32 decode loop.

TEST INFRASTRUCTURE ONLY.  Nothing in ``flux_b200`` imports this package.  It
may be imported by ``tests/``, by ``__graft_entry__.smoke()`` (as the checker)
and by ``bench.py`` (its ``cpu_baseline`` / ``--impl reference`` legs), never as
the thing measured or shipped.

Contents
--------
``smollm2``       numpy FP32 restatement of the reference path (Hugging Face
                  Llama eager as driven by Flux, plus Flux's own op oracles).
``hf_reference``  builders for the seeded Hugging Face ``LlamaForCausalLM`` that
                  the reference benchmarks as its FP32 path, and its CPU decode
                  driver used as the timed CPU baseline.
``ref_cpu``       ctypes view of the reference's own C++ CPU kernels compiled
                  by ``oracle/Makefile`` into ``oracle/_ref/`` (optional).

Parity is pinned by ``tests/golden/*.npz`` generated from the reference itself
(``tests/golden/make_golden.py``) and checked in ``tests/test_oracle.py``.
"""
