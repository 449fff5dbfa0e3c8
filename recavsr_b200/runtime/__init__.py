"""Drop-in replacements for recavsr_infer.runtime hot-path modules."""
