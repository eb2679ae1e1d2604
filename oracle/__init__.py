"""CPU oracle of OpenDecider's decision forward pass - TEST INFRASTRUCTURE.

Restatements of the reference implementation (numpy / PyTorch CPU / C) used by tests/ as the parity checker and by
bench.py as the timed CPU baseline. Nothing in the product package (opendecider_b200/) imports this package.
"""
