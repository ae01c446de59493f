"""ORACLE — test infrastructure only (CPU restatement of RusTorch's dense-contraction path)."""
