"""CPU oracle for the SLM.use token loop (test infrastructure only)."""
