"""Host CPU sizing, re-exported for the oracle's users (test infrastructure only)."""

from tests.host import limit_threads, usable_cpus  # noqa: F401
