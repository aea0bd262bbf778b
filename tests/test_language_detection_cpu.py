"""Language identification (the checks of PredictiveCoding.UnitTests/LanguageDetectionTests.cs, restated
for this package's n-gram naive-Bayes detector over profiles built from text)."""
import pytest

from predicitivecoding_b200.systems.data import LanguageDetector, LanguageProfile

PARAGRAPHS = {
    "English": "The quick brown fox jumps over the lazy dog while the children watch from the window "
               "and their parents prepare dinner in the kitchen.",
    "Italian": "Il gatto dorme sul divano mentre i bambini giocano nel giardino e la nonna prepara la cena "
               "per tutta la famiglia.",
    "French": "Le chat dort sur le canapé pendant que les enfants jouent dans le jardin et que la grand-mère "
              "prépare le dîner pour toute la famille.",
    "German": "Die Katze schläft auf dem Sofa, während die Kinder im Garten spielen und die Großmutter das "
              "Abendessen für die ganze Familie vorbereitet.",
    "Spanish": "El gato duerme en el sofá mientras los niños juegan en el jardín y la abuela prepara la cena "
               "para toda la familia.",
}


@pytest.fixture(scope="module")
def detector():
    return LanguageDetector.create_default(seed=0)


@pytest.mark.parametrize("expected", sorted(PARAGRAPHS))
def test_short_paragraphs_are_identified(detector, expected):
    assert detector.detect(PARAGRAPHS[expected]) == expected


def test_empty_or_letterless_text_is_unknown(detector):
    assert detector.detect("") == "Unknown"
    assert detector.detect("12345 !!! ??? 42") == "Unknown"


def test_detect_all_ranks_candidates_highest_first(detector):
    ranked = detector.detect_all(PARAGRAPHS["Spanish"])
    assert ranked[0].language == "Spanish"
    probs = [r.probability for r in ranked]
    assert probs == sorted(probs, reverse=True) and all(0 < p <= 1 for p in probs)


def test_same_seed_is_deterministic():
    a = LanguageDetector.create_default(seed=5).detect_all(PARAGRAPHS["German"])
    b = LanguageDetector.create_default(seed=5).detect_all(PARAGRAPHS["German"])
    assert [(r.language, r.probability) for r in a] == [(r.language, r.probability) for r in b]


def test_profiles_round_trip_in_the_langdetect_json_layout(tmp_path):
    p = LanguageProfile.from_texts("xx", ["abc abd", "abe"])
    assert p.n_words[0] == sum(v for k, v in p.freq.items() if len(k) == 1)
    path = tmp_path / "xx"
    p.save(str(path))
    q = LanguageProfile.load(str(path))
    assert (q.name, q.freq, q.n_words) == (p.name, p.freq, p.n_words)
    with pytest.raises(ValueError):
        LanguageDetector([])
