"""CPU oracle for the Engram table path: test infrastructure, never imported by the product."""
