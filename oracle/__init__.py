"""CPU oracle for the routed-expert MUL_MAT_ID path (test infrastructure only)."""
