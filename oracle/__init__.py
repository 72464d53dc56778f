"""Oracle: CPU-runnable restatement of the reference's explicit computation.

TEST INFRASTRUCTURE ONLY. Imported by tests/, __graft_entry__.smoke() and the
CPU-baseline / reference arm of bench.py, always as the checker or the timed
CPU baseline; the product package (transformer_opt) never imports it.
"""
