"""CPU oracle — TEST INFRASTRUCTURE ONLY.

A C++ restatement (vkb_oracle.cpp) of the reference's CPU algorithms on the
quantized-Whisper path, loaded with ctypes. Only tests/, __graft_entry__.smoke()
and bench.py's CPU-baseline leg may use it; the product never does.
"""
