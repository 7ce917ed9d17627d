"""CPU oracle for the Q4_0 path -- test infrastructure, never product code."""
