"""Sampling math and configuration shared with the paged engine.

Only the modules the speculative-decoding hot path imports are provided:
``specdec.sampler`` (logit post-processing, the inverse-CDF draw and the
acceptance / residual rules) and ``specdec.config`` (``SamplingConfig`` with
top-k / top-p, ``validate_gamma``).
"""
