"""Host CPU sizing, re-exported for the oracle's users (test infrastructure only)."""

from tests.host import cpu_model_name, limit_threads, usable_cpus  # noqa: F401
