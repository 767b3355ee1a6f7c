"""CPU oracle (test infrastructure only): numpy restatement of the
reference's integer semantics. Never imported by the product path."""
