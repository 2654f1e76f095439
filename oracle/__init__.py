"""CPU checkers for the paged-KV write + paged attention path (test
infrastructure; only tests, the smoke check and the benchmark's CPU-baseline
leg import this package)."""
