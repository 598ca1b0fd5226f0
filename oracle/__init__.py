"""CPU restatement of the QwenQwen3.js CPU path -- test infrastructure only (see qq3_oracle.h)."""
