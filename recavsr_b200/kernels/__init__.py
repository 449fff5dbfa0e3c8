"""Drop-in replacements for recavsr_infer.kernels."""
