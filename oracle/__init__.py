"""Test oracle for the decode-attention path (test infrastructure, not the product)."""
