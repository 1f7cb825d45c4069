"""CPU oracle and golden-fixture access for parity tests (test infrastructure only)."""
