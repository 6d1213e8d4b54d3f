"""CPU oracle (test infrastructure only): see oracle/oracle.py. The product package never imports this."""
