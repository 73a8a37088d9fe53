"""Drop-in replacements for the reference's NKI kernels (kernels/*.py) on B200.

Same function names, argument order and layouts as the reference; the NKI-only
`identity` argument is accepted and ignored, `mask` is validated as causal.
"""
