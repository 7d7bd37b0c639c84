"""CPU restatement of the reference algorithm — test infrastructure only (see ref_gpt.py)."""
