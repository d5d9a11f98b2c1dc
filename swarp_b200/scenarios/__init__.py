"""Scenario registry: the callers of the step that ``make`` can build."""

from swarp_b200.scenarios.navigation import NavigationScenario

SCENARIOS = {"navigation": NavigationScenario}


def scenario_class(name: str):
    try:
        return SCENARIOS[name]
    except KeyError:
        raise ValueError(f"unknown scenario {name!r}; valid names are {sorted(SCENARIOS)}") from None


def make_scenario(name: str, **kwargs):
    return scenario_class(name)(**kwargs)


__all__ = ["NavigationScenario", "SCENARIOS", "make_scenario", "scenario_class"]
