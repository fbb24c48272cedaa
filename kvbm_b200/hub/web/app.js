// Live view of the hub: polls its JSON routes and fills the page.
async function get(path) {
  const r = await fetch(path);
  if (!r.ok) throw new Error(path + ": " + r.status);
  return r.json();
}

function fillDl(id, obj) {
  const dl = document.getElementById(id);
  dl.replaceChildren();
  for (const [k, v] of Object.entries(obj || {})) {
    const dt = document.createElement("dt"), dd = document.createElement("dd");
    dt.textContent = k;
    dd.textContent = typeof v === "object" ? JSON.stringify(v) : String(v);
    dl.append(dt, dd);
  }
}

function fillTable(id, rows, cols) {
  const body = document.querySelector("#" + id + " tbody");
  body.replaceChildren();
  for (const row of rows) {
    const tr = body.insertRow();
    for (const c of cols) {
      const v = row[c];
      tr.insertCell().textContent = Array.isArray(v) ? v.join(",") : (v ?? "");
    }
  }
}

async function refresh() {
  const health = document.getElementById("health");
  try {
    const h = await get("/health");
    health.textContent = "healthy";
    health.className = h.status === "ok" || h.ok ? "ok" : "bad";
  } catch (e) {
    health.textContent = "unreachable";
    health.className = "bad";
    return;
  }
  const jobs = [
    get("/v1/config").then(c => fillDl("config", c)),
    get("/v1/instances").then(d => fillTable("instances", d.instances, ["instance_id", "role", "features", "address"])),
    get("/v1/indexer/config").then(c => fillDl("indexer", c)),
    get("/v1/prefill-router/targets").then(t => fillTable("targets", t.targets, ["instance_id", "inflight", "tier"])),
    get("/v1/prefill-router/counters").then(c => {
      const { calibration, ...rest } = c;
      fillDl("router", rest);
      const fmt = v => (v || []).map(x => x.toPrecision(4)).join(", ");
      fillTable("calibration", Object.entries(calibration || {}).map(([iid, m]) => ({
        iid, ts: m.ttft_samples, tc: fmt(m.ttft_coeffs), is: m.itl_samples, ic: fmt(m.itl_coeffs),
      })), ["iid", "ts", "tc", "is", "ic"]);
    }),
  ];
  await Promise.allSettled(jobs);
}

refresh();
setInterval(refresh, 2000);
