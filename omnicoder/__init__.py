"""omnicoder: a B200-native (sm_100a) framework for MoE language models.

Importing the package has no global side effects (no torch flags are changed).
"""
__version__ = "0.1.0"
