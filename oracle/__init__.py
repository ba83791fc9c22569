"""CPU oracle of the Qwen3-ASR text-decoder step (test infrastructure; see oracle.h)."""
