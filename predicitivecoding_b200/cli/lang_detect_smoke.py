"""Side-by-side language identification: random-sampling naive Bayes vs the n-gram classifier.

Reference: tools/LangDetectSmoke/Program.cs (six sentence samples, DetectAll on the Spanish one,
four short snippets).  ``--profiles DIR`` loads langdetect-format JSON profiles; without it both
detectors use the package's seed corpus.
"""
from __future__ import annotations

import sys

from ..systems.data import LanguageDetector, default_language_classifier

SAMPLES = [
    ("EN", "The committee will publish its final report on the new railway line next spring."),
    ("IT", "Il comitato pubblicherà la relazione finale sulla nuova linea ferroviaria la prossima primavera."),
    ("FR", "Le comité publiera son rapport final sur la nouvelle ligne de chemin de fer au printemps prochain."),
    ("DE", "Der Ausschuss wird seinen Abschlussbericht über die neue Bahnstrecke im nächsten Frühjahr veröffentlichen."),
    ("ES", "El comité publicará su informe final sobre la nueva línea de ferrocarril la próxima primavera."),
    ("PT", "O comitê publicará o seu relatório final sobre a nova linha ferroviária na próxima primavera."),
]
SHORT = ["¿Dónde está la biblioteca?", "Bonne nuit et à demain!", "Buona notte e a domani!", "Boa noite e até amanhã!"]


def main(argv=None) -> int:
    argv = sys.argv[1:] if argv is None else argv
    det = (LanguageDetector.from_directory(argv[argv.index("--profiles") + 1], seed=42) if "--profiles" in argv
           else LanguageDetector.create_default(seed=42))
    clf = default_language_classifier()
    print(f"{'sample':<8}{'sampling NB':<22}{'n-gram classifier':<22}")
    print("-" * 52)
    for label, text in SAMPLES:
        print(f"{label:<8}{det.detect(text):<22}{clf.predict(text):<22}")
    print("\nDetectAll (ES sample):")
    for c in det.detect_all(SAMPLES[4][1]):
        print(f"   {c.language:<12} {c.probability:.1%}")
    print("\nShort snippets (sampling NB vs n-gram classifier):")
    for t in SHORT:
        print(f"   {det.detect(t):<12} {clf.predict(t):<12} <- {t}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
