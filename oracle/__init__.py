"""CPU oracle for the DASH hot path (test infrastructure, never product code)."""
