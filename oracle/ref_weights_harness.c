/* ref_weights_harness.c -- TEST INFRASTRUCTURE ONLY. The reference's weights.c
 * (its manifest parser and pk_load_weights), compiled in place of weights.c
 * with the same flags, plus one entry point that exposes what the reference's
 * own parser (csrc/weights.c:102-207) reads for the int8 scale of named
 * entries, so the device loader's parse can be checked against it. */
#include "weights.c"

/* scales_out[i] = the scale parse_manifest gives entry names[i] (0 if absent).
 * Returns the number of manifest entries, or -1 if the file cannot be read. */
int pkref_manifest_scales(const char *json_path, const char **names, int n, float *scales_out)
{
    FILE *f = fopen(json_path, "r");
    if (!f) return -1;
    fseek(f, 0, SEEK_END);
    long len = ftell(f);
    fseek(f, 0, SEEK_SET);
    char *json = (char *)malloc(len + 1);
    if (!json) { fclose(f); return -1; }
    size_t got = fread(json, 1, len, f);
    fclose(f);
    json[got] = '\0';
    int count = 0;
    WEntry *e = parse_manifest(json, &count);
    free(json);
    if (!e) return -1;
    for (int i = 0; i < n; i++) {
        const WEntry *w = find_entry(e, count, names[i]);
        scales_out[i] = w ? w->scale : 0.0f;
    }
    for (int i = 0; i < count; i++) free((void *)e[i].name);
    free(e);
    return count;
}
