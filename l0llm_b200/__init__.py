"""l0llm_b200: a B200 (sm_100a) backend for the l0llm decoder hot path.

The compute lives in libl0b200.so (C ABI, include/l0b200.h); l0llm_b200.levelzero mirrors the
reference's LevelZeroRuntime / ComputeDevice / SharedBuffer / LlmKernelSuite / LlmModel surface on it.
"""
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
LIBRARY = PACKAGE_DIR / "libl0b200.so"
