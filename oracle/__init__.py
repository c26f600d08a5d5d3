"""CPU oracles (test infrastructure only: tests/, the smoke entry and the
bench's CPU-baseline leg use them as the checker; the product never does)."""
