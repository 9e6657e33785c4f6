"""CPU parity oracle (test infrastructure): see oracle.py and sinkslot_oracle.c."""
