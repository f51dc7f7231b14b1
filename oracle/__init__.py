"""Test oracle (CPU restatement of the reference) -- TEST INFRASTRUCTURE ONLY."""
