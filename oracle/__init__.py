"""TEST INFRASTRUCTURE ONLY: the CPU oracle (see kivi_oracle.c and oracle.py)."""
