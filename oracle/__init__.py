"""CPU oracle for the omni-tokenizer hot path -- TEST INFRASTRUCTURE ONLY (see oracle.py)."""
