"""CPU oracle (torch-eager fp32 restatement of the reference kernels) -- test infrastructure only."""
