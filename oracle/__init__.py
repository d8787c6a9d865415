"""CPU oracle for the KV-compression path (test infrastructure only)."""
