"""reng: the B200 decoder inference path of reciprocating-engine.

Host-side mirror of the reference's reng-model / reng-fp8 / reng-ceiling APIs
over libreng_cuda.so (the C ABI in include/reng_cuda.h).
"""
