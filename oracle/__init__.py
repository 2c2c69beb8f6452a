"""CPU oracle (test infrastructure only): numpy restatement of the reference's INT4 format."""
