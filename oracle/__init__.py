"""CPU parity oracle for the LeanSelect prefill hot path (test infrastructure only)."""
