"""Placeholder stand-in for timm, used ONLY by make_golden.py.

The reference routing modules import a handful of timm names at module level
(classes they subclass or reference, a registry decorator, data constants).
None of them is on the routing path this fixture generator exercises, so each
name here is an inert placeholder written for this repository.  This is not
timm and is never imported by the product or by tests.
"""
