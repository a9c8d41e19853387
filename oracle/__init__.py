"""CPU oracle (test infrastructure only): restatements of the reference's quantized-linear
arithmetic, used by tests, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py`."""
