"""CPU oracle and reference builds -- test infrastructure, never product code."""
