"""CPU oracle for the Block-RVQ runtime linear (test infrastructure only; never imported by the product)."""
