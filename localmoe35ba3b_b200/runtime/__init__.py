"""Runtime kernels driving the operators: routing metadata, prefill expert FFN, decode."""
