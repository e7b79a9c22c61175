"""TEST INFRASTRUCTURE -- the CPU oracle for darknet-zig's array ops (see oracle.py).

Imported only by tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg."""
