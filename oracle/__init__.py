"""CPU oracle for the deformable convolution (test infrastructure only)."""
