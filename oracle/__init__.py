"""CPU checker package: the oracle restatement (oracle.py, gpt2.py) and the
reference's own CPU path (_ref).  Test infrastructure only."""
