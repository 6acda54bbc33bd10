"""CPU oracles for parity testing -- TEST INFRASTRUCTURE ONLY.

ref_f64   float64 numpy restatement of reference.py (the precision oracle)
ref_torch PyTorch-on-CPU restatement in the input dtype (the reference's CPU
          path, timed as the CPU baseline)

Only tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / reference
arm may import this package; the product (autokernel_b200) never does.
"""
