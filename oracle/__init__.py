"""CPU parity checkers (test infrastructure only; see nfo_oracle.c and ref_shim.cpp)."""
