"""CPU oracle for the hot/cold sparse-FFN path (test infrastructure only)."""
