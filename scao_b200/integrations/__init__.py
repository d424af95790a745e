"""Framework integrations of the scao_b200 optimizer."""
