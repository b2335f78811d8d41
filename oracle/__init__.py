"""CPU oracle of the llama2c hot path -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, as the checker or the timed CPU baseline. The product
(libce_b200.so and the cuda-elastic_b200 package) never imports it.
"""
