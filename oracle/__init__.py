"""Test infrastructure only: the CPU oracle for the attention path (see attention_oracle)."""
