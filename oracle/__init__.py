"""CPU oracle for rich-triplet's Q4_K decode path -- test infrastructure only."""
