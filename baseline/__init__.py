"""The comparison arm: the reference's own ``qtts`` package, installed unmodified.

``baseline/_ref`` holds the reference installed by :func:`baseline.install.install`
(an offline ``pip install --target``, git-ignored). Only the benchmark's comparison
sections and the tests import it; the library (``qtts_b200``) never does.
"""
