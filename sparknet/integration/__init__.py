"""Engine integrations."""
