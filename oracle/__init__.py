"""CPU parity checker for the EXL3 trellis quantizer (test infrastructure only;
see exl3_oracle.py)."""
